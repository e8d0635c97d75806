"""ctypes binding of libkvb.so (the C ABI declared in include/kvb.h).

The library is built in-tree by ``python -m kernelverse_b200.build``.  There is
no fallback: if the shared library is missing, importing the product path
raises, so nothing can silently run on the CPU or through PyTorch instead.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

LIB_PATH = Path(os.environ.get("KVB_LIB", Path(__file__).resolve().parent / "libkvb.so"))

# status / dtype codes (include/kvb.h)
OK = 0
F32, F16, BF16, I8, U8, I32, I64, E4M3 = range(8)

_P, _I, _I64, _F, _SZ = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float, ctypes.c_size_t

# name -> (restype, argtypes); must mirror include/kvb.h exactly
SIGNATURES = {
    "kvb_last_error": (ctypes.c_char_p, []),
    "kvb_abi_version": (_I, []),
    "kvb_device_status": (ctypes.c_uint, [_I]),
    "kvb_check_device": (_I, [_I]),
    "kvb_set_wait_limit_ns": (_I, [ctypes.c_uint64]),
    "kvb_selftest_wait_timeout": (_I, [_P, _P, _P]),
    "kvb_selftest_div_rn": (_I, [_P, _P, _P, _I64, _P]),
    "kvb_dynamic_scaled_int8_quant_workspace_size": (_SZ, []),
    "kvb_dynamic_scaled_int8_quant": (_I, [_P, _I, _I64, _P, _P, _P, _P, _SZ, _P]),
    "kvb_per_token_group_quant_int8": (_I, [_P, _I, _I64, _I64, _I64, _F, _P, _P, _P]),
    "kvb_static_scaled_int8_quant": (_I, [_P, _I, _I64, _P, _P, _P, _P]),
    "kvb_add_rmsnorm": (_I, [_P, _P, _P, _I, _I64, _I64, _F, _P, _P]),
    "kvb_add_rmsnorm_quant": (_I, [_P, _P, _P, _I, _I64, _I64, _F, _P, _P, _I, _P, _P]),
    "kvb_w8a8_workspace_size": (_SZ, [_I64, _I64, _I64, _I, _I]),
    "kvb_w8a8_scaled_mm": (_I, [_P, _P, _I, _P, _P, _P, _I, _P, _P, _I64, _I64, _I64, _P, _I, _I64, _P, _SZ, _P]),
    "kvb_w8a8_scaled_mm_allgather": (_I, [_P, _P, _P, _P, _P, _I, _I64, _I64, _I64, _P, _I, _I, _I64, _I, _P]),
    "kvb_w8a8_scaled_mm_act": (_I, [_P, _P, _P, _P, _P, _I, _I64, _I64, _I64, _I, _P, _I, _I64, _P]),
    "kvb_w8a8_scaled_mm_act_allgather": (_I, [_P, _P, _P, _P, _P, _I, _I64, _I64, _I64, _I, _P, _I, _I, _I64, _I, _P]),
    "kvb_paged_kv_cache_update": (_I, [_P, _P, _P, _P, _I, _I, _I64, _I64, _I64, _P]),
    "kvb_paged_fp8_kv_write": (_I, [_P, _I, _P, _P, _I, _P, _I64, _I64, _I, _I, _P]),
    "kvb_kv_cache_write": (_I, [_P, _P, _P, _P, _P, _P, _P, _I, _I, _I, _I64, _I64, _I64, _I64, _I64, _P]),
    "kvb_paged_attention_workspace_size": (_SZ, [_I, _I, _I, _I]),
    "kvb_paged_attention_auto_partition": (_I, [_I, _I64]),
    "kvb_flash_attn_with_kvcache_workspace_size": (_SZ, [_I, _I, _I, _I, _I64]),
    "kvb_flash_attn_with_kvcache": (_I, [_P, _P, _P, _I, _P, _I, _I, _I, _I64, _I, _I, _I, _F, _P, _P, _P, _SZ, _P]),
    "kvb_paged_attention": (_I, [_P, _I, _P, _P, _I, _P, _P, _P, _I, _P, _I64, _I, _I, _I, _I, _I, _I64, _I64, _F,
                                 _P, _P, _I, _I, _P, _I, _P, _P, _P, _I, _P, _SZ, _P]),
    "kvb_batched_prefill_attention": (_I, [_P, _P, _P, _I, _P, _P, _I, _I64, _I64, _I, _I, _I, _F, _P, _P]),
    "kvb_batched_prefill_attention_variant": (_I, [_P, _P, _P, _I, _P, _P, _I, _I64, _I64, _I, _I, _I, _F, _P, _I,
                                                   _P]),
    "kvb_paged_attention_noalloc": (_I, [_P, _I, _P, _P, _I, _P, _P, _P, _I, _P, _I64, _I, _I, _I, _I, _I, _I64, _I64,
                                         _F, _P, _P, _I, _I, _P, _I, _P, _P, _P, _I, _P]),
}


class KvbError(RuntimeError):
    """A libkvb entry point returned a non-zero status."""

    def __init__(self, fn: str, code: int, msg: str):
        super().__init__(f"{fn} failed with status {code}: {msg}")
        self.code = code


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is not built; run `python -m kernelverse_b200.build` "
                               "(kernelverse_b200 has no CPU or PyTorch fallback)")
        h = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            f = getattr(h, name)
            f.restype, f.argtypes = res, args
        _lib = h
    return _lib


def call(name: str, *args) -> None:
    rc = getattr(lib(), name)(*args)
    if rc != OK:
        raise KvbError(name, rc, lib().kvb_last_error().decode(errors="replace"))


def check_device(reset: bool = True) -> None:
    """Synchronise the current device and raise KvbError if a bounded device-side wait gave up
    (KVB_E_TIMEOUT) or an out-of-range index was skipped (KVB_E_INDEX) since the last reset."""
    call("kvb_check_device", 1 if reset else 0)
