"""CPU oracle for the W8A8 int8 GEMM rows (test infrastructure only).

* ``w8a8_acc``: the exact int32 accumulator ``A[M,K] @ B[N,K]^T``.  It is
  evaluated as a float64 BLAS product, which is exact here because every
  partial sum is an integer below 2**53 (|acc| <= K * 127**2).
* ``w8a8_scaled_mm``: the BASELINE third config epilogue
  ``out = (float32(acc) * sa[m]) * sb[n] + bias[n]`` in float32, rounded to the
  output dtype.  Each operation is a separate float32 rounding, the same order
  the device epilogue uses, so bf16 outputs are expected bit-exact.
* ``int8_scaled_mm_azp``: ``operators/gemm/int8_scaled_mm_azp/int8_scaled_mm_azp.py:61-85``
  -- ``(a*sa) @ ((b - azp)*sb) + azp_adj [+ bias]`` with ``b`` laid out
  ``[K, N]``; ``azp_adj`` is always added (``:82``).  The oracle evaluates it
  in float64 (the reference uses float32, so the two agree to float32
  rounding, well inside the reference's tolerances).
"""
from __future__ import annotations

import numpy as np

from .numerics import round_to


def w8a8_acc(a: np.ndarray, b_nk: np.ndarray) -> np.ndarray:
    acc = np.asarray(a, np.float64) @ np.asarray(b_nk, np.float64).T
    return acc.astype(np.int64).astype(np.int32)


def w8a8_scaled_mm(a, b_nk, sa, sb, bias=None, out_dtype: str = "BF16", acc=None) -> np.ndarray:
    if acc is None:
        acc = w8a8_acc(a, b_nk)
    out = (acc.astype(np.float32) * np.asarray(sa, np.float32)[:, None]).astype(np.float32)
    out = (out * np.asarray(sb, np.float32)[None, :]).astype(np.float32)
    if bias is not None:
        out = (out + np.asarray(bias, np.float32)[None, :]).astype(np.float32)
    return round_to(out, out_dtype)


def int8_scaled_mm_azp(a, b_kn, a_scales, b_scales, azp_adj, azp, bias,
                       has_azp: bool, has_bias: bool, out_dtype: str) -> np.ndarray:
    a64 = np.asarray(a, np.float64) * np.asarray(a_scales, np.float64).reshape(-1, 1)
    b64 = np.asarray(b_kn, np.float64)
    if has_azp:
        b64 = b64 - np.asarray(azp, np.float64).reshape(1, -1)
    b64 = b64 * np.asarray(b_scales, np.float64).reshape(1, -1)
    out = a64 @ b64 + np.asarray(azp_adj, np.float64).reshape(1, -1)
    if has_bias:
        out = out + np.asarray(bias, np.float64).reshape(1, -1)
    return round_to(out.astype(np.float32), out_dtype)
