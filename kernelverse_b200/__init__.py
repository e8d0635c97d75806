"""kernelverse_b200 -- B200-native (sm_100a) kernels for KernelVerse's quantised decoder-layer hot path.

``kernelverse_b200.ops`` holds one function per reference operator on the path;
``kernelverse_b200.drop_in`` holds the ``ModelNew`` files that KernelVerse's
``cuda`` backend executes.  All compute runs in ``libkvb.so`` (built in-tree by
``python -m kernelverse_b200.build``); there is no CPU fallback.
"""
from ._lib import KvbError, LIB_PATH  # noqa: F401

__all__ = ["KvbError", "LIB_PATH"]
