"""Make KernelVerse's operator registry discover this repository's operator packages.

KernelVerse discovers operators only under its own ``operators/`` directory
(``discover_operator_specs``, operators/registry.py:79-100) and caches the result with
``lru_cache``.  ``install()`` wraps ``discover_operator_specs`` so that the packages under
``kernelverse_b200/operators/<category>/<op>/`` are merged in (reference packages win on a
name clash); ``get_operator_spec`` (:103-111) looks the function up at call time, and
``load_module`` / ``load_object`` (:172-203) load files outside the reference root by path.

Evaluations run in spawned processes (runner/generated_correctness_runner.py:1089-1121),
so the overlay must be active in every interpreter: put ``kernelverse_b200/overlay_site``
on ``PYTHONPATH``; its ``sitecustomize`` calls ``install_import_hook()``, which patches the
registry module the moment it is first imported.
"""
from __future__ import annotations

import importlib.abc
import importlib.util
import sys
from functools import lru_cache
from pathlib import Path

OPERATORS_ROOT = Path(__file__).resolve().parent / "operators"
_REQUIRED = ("shapes.py", "config.json", "docs.md", "helpers.py")


def local_packages():
    """(category, op_dir) of every package here that follows the reference's convention."""
    out = []
    for cat in sorted(p for p in OPERATORS_ROOT.iterdir() if p.is_dir() and not p.name.startswith(("_", "."))):
        for op in sorted(p for p in cat.iterdir() if p.is_dir() and not p.name.startswith(("_", "."))):
            if (op / f"{op.name}.py").exists() and all((op / f).exists() for f in _REQUIRED):
                out.append((cat.name, op))
    return out


def install(registry=None) -> None:
    """Patch a loaded ``operators.registry`` module in place (idempotent)."""
    if registry is None:
        import operators.registry as registry  # noqa: F811  (the reference's module)
    if getattr(registry, "_kvb_overlay", False):
        return
    original = registry.discover_operator_specs

    @lru_cache(maxsize=1)
    def discover_operator_specs():
        specs = dict(original())
        for category, op_dir in local_packages():
            specs.setdefault(op_dir.name, registry._build_spec(category, op_dir))
        return specs

    registry.discover_operator_specs = discover_operator_specs
    registry._kvb_overlay = True


class _RegistryHook(importlib.abc.MetaPathFinder, importlib.abc.Loader):
    """Runs ``install`` right after ``operators.registry`` is executed."""

    def find_spec(self, fullname, path, target=None):
        if fullname != "operators.registry":
            return None
        for finder in sys.meta_path:
            if finder is self:
                continue
            spec = finder.find_spec(fullname, path, target) if hasattr(finder, "find_spec") else None
            if spec is not None:
                self._inner = spec.loader
                spec.loader = self
                return spec
        return None

    def create_module(self, spec):
        return self._inner.create_module(spec) if hasattr(self._inner, "create_module") else None

    def exec_module(self, module):
        self._inner.exec_module(module)
        install(module)


def install_import_hook() -> None:
    if "operators.registry" in sys.modules:
        install(sys.modules["operators.registry"])
        return
    if not any(isinstance(f, _RegistryHook) for f in sys.meta_path):
        sys.meta_path.insert(0, _RegistryHook())
