"""Bit-level number formats for the CPU oracle (test infrastructure only).

This module is part of the parity oracle.  Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may import it;
the CUDA product path never does.

numpy has no bfloat16 or float8 types, so low-precision tensors are carried as
float32 arrays whose values are exactly representable in the named format,
plus helpers that round float32 values to that format the way PyTorch's casts
do (round-to-nearest-even):

* bf16:  ``Tensor.to(torch.bfloat16)``  (PyTorch, c10/util/BFloat16.h semantics)
* fp16:  IEEE binary16, numpy's own cast
* e4m3fn: ``Tensor.to(torch.float8_e4m3fn)`` -- the OCP FP8 E4M3 format with
  bias 7, no infinities, one NaN pattern per sign (S.1111.111), max finite 448,
  subnormals m * 2**-9.  The encoder here is written from that format
  definition; ``tests/test_oracle_numerics.py`` checks it against torch's cast
  over every float32 that rounds to each code boundary.
"""
from __future__ import annotations

import numpy as np

E4M3_MAX = 448.0
INT8_QMAX = 127.0
# The reference's minimum scale (operators/quantization/dynamic_scaled_int8_quant/helpers.py:8).
MIN_SCALING_FACTOR = np.float32(1.0 / (448.0 * 512.0))


# ----------------------------------------------------------------------------- bf16
def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns (uint16), round-to-nearest-even, NaN kept quiet."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) >> 16) & 0xFFFF
    r = np.where(nan, ((u >> 16) | 0x40) & 0xFFFF, r)
    return r.astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_bf16(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bf16 value (returned as float32)."""
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


def round_fp16(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round float32 values to ``dtype`` in {"FP32","FP16","BF16"} (float32 result)."""
    dtype = dtype.upper()
    x = np.asarray(x, dtype=np.float32)
    if dtype == "FP32":
        return x
    if dtype == "FP16":
        return round_fp16(x)
    if dtype == "BF16":
        return round_bf16(x)
    raise ValueError(f"unsupported dtype {dtype}")


# ----------------------------------------------------------------------------- e4m3fn
def e4m3_encode(x: np.ndarray) -> np.ndarray:
    """float32 -> e4m3fn codes (uint8), round-to-nearest-even.

    Inputs must already be finite and within [-448, 448] (every caller clamps
    first, exactly as the reference-side composition does before its cast).
    A normal value a = 2**e * (1 + m/8) has code (e+7)<<3 | m; a subnormal
    a = m * 2**-9 has code m.  Both are covered by q = rint(a / 2**(e-3)) with
    e = max(floor(log2 a), -6), code = ((e+7)<<3) + q - 8, where q == 16
    carries into the next binade automatically.
    """
    x = np.asarray(x, dtype=np.float32)
    if np.any(~np.isfinite(x)) or np.any(np.abs(x) > E4M3_MAX):
        raise ValueError("e4m3_encode expects finite values clamped to +-448")
    a = np.abs(x).astype(np.float64)
    sign = np.signbit(x)
    _, exp = np.frexp(a)            # a = mant * 2**exp with mant in [0.5, 1)
    e = np.maximum(exp.astype(np.int64) - 1, -6)
    q = np.rint(a / np.exp2((e - 3).astype(np.float64)))
    code = ((e + 7) << 3) + q.astype(np.int64) - 8
    code = np.where(a == 0, 0, code)
    code = code | (sign.astype(np.int64) << 7)
    return code.astype(np.uint8)


def e4m3_decode(c: np.ndarray) -> np.ndarray:
    """e4m3fn codes (uint8) -> float32 values (NaN for S.1111.111)."""
    c = np.asarray(c, dtype=np.uint8).astype(np.int64)
    s = np.where(c & 0x80, -1.0, 1.0)
    e = (c >> 3) & 0xF
    m = c & 0x7
    val = np.where(e == 0, m * 2.0 ** -9, (1.0 + m / 8.0) * np.exp2(e - 7.0))
    val = np.where((e == 15) & (m == 7), np.nan, val)
    return (s * val).astype(np.float32)


def e4m3_ordinal(c: np.ndarray) -> np.ndarray:
    """Map e4m3 codes to a signed integer line so that |ord(a)-ord(b)| counts ulps."""
    c = np.asarray(c, dtype=np.uint8).astype(np.int64)
    mag = c & 0x7F
    return np.where(c & 0x80, -mag, mag)


def e4m3_quantize(y: np.ndarray, scale: np.ndarray) -> np.ndarray:
    """codes = e4m3(clamp(y / scale, -448, 448)) with an IEEE float32 division."""
    q = np.asarray(y, dtype=np.float32) / np.asarray(scale, dtype=np.float32)
    return e4m3_encode(np.clip(q, -E4M3_MAX, E4M3_MAX).astype(np.float32))
