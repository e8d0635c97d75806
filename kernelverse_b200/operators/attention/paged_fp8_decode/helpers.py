"""Helpers for paged_fp8_decode."""
from typing import Any, Dict

REQUIRED_SHAPE_KEYS = ("batch_size", "num_q_heads", "num_kv_heads", "head_dim", "block_size", "min_context",
                       "max_context")
E4M3_MAX = 448.0


def validate_shape(shape: Dict[str, Any]) -> None:
    missing = [k for k in REQUIRED_SHAPE_KEYS if k not in shape]
    if missing:
        raise ValueError(f"Missing shape parameter(s): {', '.join(missing)}")
    for k in REQUIRED_SHAPE_KEYS:
        if int(shape[k]) <= 0:
            raise ValueError(f"{k} must be positive.")
    if int(shape["num_q_heads"]) % int(shape["num_kv_heads"]):
        raise ValueError("num_q_heads must be divisible by num_kv_heads.")
    if int(shape["min_context"]) > int(shape["max_context"]):
        raise ValueError("min_context must not exceed max_context.")
