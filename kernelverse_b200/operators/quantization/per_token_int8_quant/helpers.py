"""Helpers for per_token_int8_quant."""
from typing import Any, Dict

import torch

REQUIRED_SHAPE_KEYS = ("num_tokens", "hidden_dim", "dtype")
DTYPE_NAME_MAP = {"FP32": torch.float32, "FP16": torch.float16, "BF16": torch.bfloat16}
INT8_QMAX = 127.0
EPS = 1e-6


def validate_shape(shape: Dict[str, Any]) -> None:
    missing = [k for k in REQUIRED_SHAPE_KEYS if k not in shape]
    if missing:
        raise ValueError(f"Missing shape parameter(s): {', '.join(missing)}")
    for k in ("num_tokens", "hidden_dim"):
        if int(shape[k]) <= 0:
            raise ValueError(f"{k} must be positive.")
    _resolve_dtype(shape["dtype"])


def _resolve_dtype(name: str) -> torch.dtype:
    if name not in DTYPE_NAME_MAP:
        raise ValueError(f"Unsupported dtype: {name}")
    return DTYPE_NAME_MAP[name]
