"""Operator packages for the BASELINE variants of the hot path that have no KernelVerse
operator, in KernelVerse's package convention (``<op>.py`` with ``Model`` and
``generate_inputs``, ``shapes.py``, ``config.json``, ``docs.md``, ``helpers.py``;
operators/registry.py:14,39-76).  ``kernelverse_b200.registry_overlay`` makes the reference
registry discover them next to its own packages.  Each ``Model`` is the PyTorch statement of
the operator -- the baseline the harness compares ``ModelNew`` against -- and its
``ModelNew`` lives in ``kernelverse_b200/drop_in/``.
"""
from pathlib import Path

ROOT = Path(__file__).resolve().parent
