"""Install the unmodified reference (KernelVerse) into ``baseline/_ref``.

    python baseline/install_ref.py [--src REFERENCE_TREE]

``bench.py --impl reference`` and the GPU test of the reference's own correctness runner
import the reference from ``baseline/_ref`` (git-ignored; it travels to the GPU box with the
working tree, like the built ``libkvb.so``).  The reference tree has neither ``setup.py`` nor
``pyproject.toml``, so ``pip install`` refuses it as it stands.  This recipe copies the tree
to a temporary directory, adds a ``pyproject.toml`` that declares its six top-level packages
(``operators``, ``runner``, ``backends``, ``utils``, ``evaluator``, ``codegen``; most
operator directories are namespace packages) and their data files, and runs the offline
install

    python -m pip install --no-index --no-build-isolation --find-links /opt/wheelhouse \
        --no-deps --target baseline/_ref <copy>

No reference source file is changed.  ``--no-deps``: the reference's ``requirements.txt``
lists only torch and numpy (unpinned), which are already installed.  The source tree
defaults to the ``KV_REFERENCE_ROOT`` environment variable.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent
TARGET = HERE / "_ref"
PACKAGES = ("operators", "runner", "backends", "utils", "evaluator", "codegen")

PYPROJECT = """\
[build-system]
requires = ["setuptools>=61"]
build-backend = "setuptools.build_meta"

[project]
name = "kernelverse-reference"
version = "0.0.0"

[tool.setuptools.packages.find]
where = ["."]
include = [{includes}]
namespaces = true

[tool.setuptools.package-data]
"*" = ["*.json", "*.md", "*.txt", "*.cpp", "*.hpp", "*.h", "*.sh", "*.example"]
"""


def install(src: Path, target: Path = TARGET) -> Path:
    if not (src / "operators" / "registry.py").exists():
        raise SystemExit(f"{src} is not a KernelVerse tree (operators/registry.py missing)")
    with tempfile.TemporaryDirectory(prefix="kv_ref_") as tmp:
        copy = Path(tmp) / "kernelverse"
        shutil.copytree(src, copy, ignore=shutil.ignore_patterns("__pycache__", "*.pyc", ".git"))
        includes = ", ".join(f'"{p}", "{p}.*"' for p in PACKAGES)
        (copy / "pyproject.toml").write_text(PYPROJECT.format(includes=includes))
        if target.exists():
            shutil.rmtree(target)
        cmd = [sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation", "--find-links",
               "/opt/wheelhouse", "--no-deps", "--target", str(target), str(copy)]
        subprocess.run(cmd, check=True)
    (target / "INSTALLED_FROM.txt").write_text(f"{src}\n")
    return target


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--src", default=os.environ.get("KV_REFERENCE_ROOT"))
    a = ap.parse_args()
    if not a.src:
        raise SystemExit("give --src or set KV_REFERENCE_ROOT to the reference tree")
    print(install(Path(a.src)))


if __name__ == "__main__":
    main()
