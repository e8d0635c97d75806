"""Helpers for add_rmsnorm_fp8_quant."""
from typing import Any, Dict

import torch

REQUIRED_SHAPE_KEYS = ("shape", "eps", "dtype")
DTYPE_NAME_MAP = {"FP32": torch.float32, "FP16": torch.float16, "BF16": torch.bfloat16}
E4M3_MAX = 448.0
# operators/quantization/dynamic_scaled_int8_quant/helpers.py:8 in the KernelVerse tree
MIN_SCALING_FACTOR = 1.0 / (448.0 * 512.0)


def validate_shape(shape: Dict[str, Any]) -> None:
    missing = [k for k in REQUIRED_SHAPE_KEYS if k not in shape]
    if missing:
        raise ValueError(f"Missing shape parameter(s): {', '.join(missing)}")
    dims = shape["shape"]
    if not isinstance(dims, (list, tuple)) or not dims or any(int(d) <= 0 for d in dims):
        raise ValueError("shape must be a non-empty list of positive integers.")
    if float(shape["eps"]) <= 0:
        raise ValueError("eps must be positive.")
    _resolve_dtype(shape["dtype"])


def _resolve_dtype(name: str) -> torch.dtype:
    if name not in DTYPE_NAME_MAP:
        raise ValueError(f"Unsupported dtype: {name}")
    return DTYPE_NAME_MAP[name]
