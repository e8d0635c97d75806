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
* ``w8a8_scaled_mm_act``: the gate+up GEMM followed by SwiGLU
  (``operators/activation/swiglu/swiglu.py:24-28``) or mul-and-silu
  (``operators/activation/mul_and_silu/mul_and_silu.py:24-29``) on the GEMM's
  stored (rounded) output, in float32.
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


def silu_f32(x: np.ndarray) -> np.ndarray:
    """x / (1 + e^-x) in float32 (each operation rounded to float32)."""
    x = np.asarray(x, np.float32)
    with np.errstate(over="ignore"):
        return (x / (np.float32(1.0) + np.exp(-x))).astype(np.float32)


def w8a8_scaled_mm_act(a, b_first, b_second, sa, s_first, s_second, bias_first=None, bias_second=None,
                       act: str = "swiglu", out_dtype: str = "BF16") -> np.ndarray:
    """The W8A8 GEMM of each operand weight rounded to ``out_dtype`` (what the unfused GEMM
    stores), then operators/activation/swiglu/swiglu.py:24-28 (``silu(first) * second``) or
    operators/activation/mul_and_silu/mul_and_silu.py:24-29 (``first * silu(second)``) in
    float32, rounded to ``out_dtype``."""
    f = round_to(w8a8_scaled_mm(a, b_first, sa, s_first, bias_first, "FP32"), out_dtype).astype(np.float32)
    g = round_to(w8a8_scaled_mm(a, b_second, sa, s_second, bias_second, "FP32"), out_dtype).astype(np.float32)
    y = silu_f32(f) * g if act == "swiglu" else f * silu_f32(g)
    return round_to(y.astype(np.float32), out_dtype)

