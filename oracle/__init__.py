"""CPU parity oracle for the quantised decoder-layer hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the reference KernelVerse operators that the
B200 kernels replace (each function cites the reference file:line it follows).
It is the checker, never the product: only ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU-baseline leg (``--impl reference`` and the
``cpu_baseline`` field) may import it.  The CUDA path in ``kernelverse_b200``
never imports it and fails loudly when its extension is missing.

Pinning: ``tests/test_oracle_golden.py`` checks every function here against
fixtures in ``tests/golden/`` that ``tests/golden/make_golden.py`` produced by
running the reference's own ``Model.forward`` on CPU (torch 2.11.0), and
``tests/test_oracle_numerics.py`` checks the e4m3 encoder against the format
definition and torch's cast.
"""
from . import attention, gemm, kv_cache, numerics, quant, rmsnorm  # noqa: F401
