"""Drop-in ``ModelNew`` files for KernelVerse's ``cuda`` backend.

Each ``<operator>.py`` here is a complete generated-code file in the form KernelVerse's
``CudaBackend.compile`` executes (backends/cuda_backend.py:35-45): it defines ``ModelNew``
with the reference ``Model``'s constructor and ``forward`` signature and runs the operator
on the B200 kernels through ``kernelverse_b200.ops``.  ``path(op_name)`` returns the file to
hand to ``python -m evaluator.main --generated-path``.
"""
from pathlib import Path

HERE = Path(__file__).resolve().parent


def path(op_name: str) -> Path:
    p = HERE / f"{op_name}.py"
    if not p.exists():
        raise FileNotFoundError(f"no drop-in ModelNew for {op_name}")
    return p


def available():
    return sorted(p.stem for p in HERE.glob("*.py") if p.stem != "__init__")
