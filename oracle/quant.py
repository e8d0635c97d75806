"""CPU oracle for the int8 quantisation rows of the hot path (test infrastructure only).

Restates, in numpy, the reference operators

* ``operators/quantization/dynamic_scaled_int8_quant/dynamic_scaled_int8_quant.py:21-26``
  (per-tensor scale, computed in the input dtype, clamped at MIN_SCALING_FACTOR;
  constants at ``.../helpers.py:7-8``), and
* ``operators/quantization/per_token_group_quant_int8/per_token_group_quant_int8.py:23-32``
  (per-(token, group) fp32 scale, ``clamp_min(eps)``), and
* ``operators/quantization/static_scaled_int8_quant/static_scaled_int8_quant.py:28-32``
  (static scale and zero point; MIN_SCALE at ``.../helpers.py:8``), in its float32
  correctness mode.

Low-precision inputs are float32 arrays holding exactly representable values
(see ``oracle.numerics``).  Only tests, ``smoke()`` and ``bench.py``'s CPU
baseline may call this module.
"""
from __future__ import annotations

import numpy as np

from .numerics import INT8_QMAX, MIN_SCALING_FACTOR, round_to


def dynamic_scaled_int8_quant(x: np.ndarray, dtype: str):
    """Per-tensor dynamic int8 quantisation.

    Follows dynamic_scaled_int8_quant.py:22-26: ``amax(|x|)`` in the input dtype
    (exact: it is one of the inputs), ``/127`` evaluated in float32 and rounded
    back to the input dtype, widened to float32, clamped below at
    MIN_SCALING_FACTOR; then ``q = round_half_even(clamp(x / scale, -127, 127))``.
    Returns ``(q int8, scale float32[1], azp int32[1])``.  A 1-D input yields a
    ``[1, n]`` q, exactly as the reference's broadcast against a ``[1, 1]`` scale does.
    """
    x = np.asarray(x, dtype=np.float32)
    amax = np.float32(np.max(np.abs(x))) if x.size else np.float32(0.0)
    s = round_to(np.array([amax / np.float32(INT8_QMAX)], dtype=np.float32), dtype)
    scale = np.maximum(s.astype(np.float32), MIN_SCALING_FACTOR).astype(np.float32)
    q = np.rint(np.clip(x / scale[0], -INT8_QMAX, INT8_QMAX)).astype(np.int8)
    if x.ndim == 1:
        q = q.reshape(1, -1)
    return q, scale.reshape(1), np.zeros((1,), dtype=np.int32)


def per_token_group_quant_int8(x: np.ndarray, group_size: int, eps: float):
    """Per-token, per-group int8 quantisation (per_token_group_quant_int8.py:24-32).

    ``scale[t, g] = max(amax(|x[t, g*G:(g+1)*G]|) / 127, eps)`` in float32 and
    ``q = clamp(round_half_even(x / scale), -127, 127)``.  With ``group_size ==
    hidden`` this is the per-token quantisation of the first BASELINE config.
    Returns ``(q int8 [T, H], scales float32 [T, H // group_size])``.
    """
    x = np.asarray(x, dtype=np.float32)
    t, h = x.shape
    g = h // group_size
    grouped = x.reshape(t, g, group_size)
    amax = np.max(np.abs(grouped), axis=-1) if group_size else np.zeros((t, g), np.float32)
    scales = np.maximum(amax.astype(np.float32) / np.float32(INT8_QMAX), np.float32(eps)).astype(np.float32)
    q = np.clip(np.rint(grouped / scales[..., None]), -INT8_QMAX, INT8_QMAX).astype(np.int8)
    return q.reshape(t, h), scales


def static_scaled_int8_quant(x: np.ndarray, scale, azp=0):
    """Static-scale int8 quantisation (static_scaled_int8_quant.py:28-32, float32 mode):
    ``q = clamp(round_half_even(x / max(scale, MIN_SCALE) + azp), -127, 127)`` with the
    quotient and the sum each rounded to float32.  Returns int8 of x's shape."""
    x = np.asarray(x, dtype=np.float32)
    s = np.maximum(np.float32(np.asarray(scale, np.float32).reshape(-1)[0]), MIN_SCALING_FACTOR).astype(np.float32)
    z = np.float32(np.asarray(azp).reshape(-1)[0])
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        centered = (x / s).astype(np.float32) + z
    return np.clip(np.rint(centered), -INT8_QMAX, INT8_QMAX).astype(np.int8)

