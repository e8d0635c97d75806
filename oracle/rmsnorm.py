"""CPU oracle for residual-add + RMSNorm (+ per-row quantisation) (test infrastructure only).

Restates ``operators/normalization/add_rmsnorm/add_rmsnorm.py:24-35`` in its
"correctness" compute mode (float32 intermediates, ``:17-22``): ``s = x + r``,
``y = (s * rsqrt(mean(s**2) + eps)) * w``, cast to the output dtype.

The fused BASELINE variant (second config) additionally returns the updated
residual ``bf16(s)`` and quantises ``y`` per row: ``scale = max(amax|y| / Q,
MIN_SCALING_FACTOR)`` and ``codes = quant(y / scale)`` with Q = 448 for e4m3fn
(clamped to +-448 before the cast) or Q = 127 for int8 (round-half-even, clamped
to +-127).  There is no reference operator for the fused form; it composes the
reference's add_rmsnorm with the reference's own quantisation constants
(``operators/quantization/dynamic_scaled_int8_quant/helpers.py:7-8``).

The mean of squares is accumulated in float64 and rounded once to float32;
the device kernel sums in float32 in another order, so ``y`` agrees to a few
float32 ulps (tests state the tolerance).
"""
from __future__ import annotations

import numpy as np

from .numerics import E4M3_MAX, INT8_QMAX, MIN_SCALING_FACTOR, e4m3_quantize, round_bf16, round_to


def _normalize(x: np.ndarray, r: np.ndarray, w: np.ndarray, eps: float):
    s = np.asarray(x, np.float32) + np.asarray(r, np.float32)
    var = np.mean(s.astype(np.float64) ** 2, axis=-1, keepdims=True).astype(np.float32)
    rinv = (np.float32(1.0) / np.sqrt(var + np.float32(eps))).astype(np.float32)
    y = ((s * rinv).astype(np.float32) * np.asarray(w, np.float32)).astype(np.float32)
    return s, y


def add_rmsnorm(x, r, w, eps: float, dtype: str) -> np.ndarray:
    """Reference add_rmsnorm (correctness mode) -> values rounded to ``dtype``."""
    _, y = _normalize(x, r, w, eps)
    return round_to(y, dtype)


def add_rmsnorm_quant(x, r, w, eps: float, code_kind: str = "e4m3"):
    """Fused add + RMSNorm + per-row quantisation (BASELINE second config).

    Returns ``(residual_out bf16-valued float32, codes, scales float32[rows], y float32)``
    where codes are uint8 e4m3fn patterns (``code_kind == "e4m3"``) or int8.
    """
    s, y = _normalize(x, r, w, eps)
    r_out = round_bf16(s)
    amax = np.max(np.abs(y), axis=-1, keepdims=True).astype(np.float32)
    qmax = np.float32(E4M3_MAX if code_kind == "e4m3" else INT8_QMAX)
    scales = np.maximum(amax / qmax, MIN_SCALING_FACTOR).astype(np.float32)
    if code_kind == "e4m3":
        codes = e4m3_quantize(y, scales)
    elif code_kind == "int8":
        codes = np.clip(np.rint(y / scales), -INT8_QMAX, INT8_QMAX).astype(np.int8)
    else:
        raise ValueError(code_kind)
    return r_out, codes, scales[..., 0], y
