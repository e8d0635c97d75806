"""Helpers for w8a8_scaled_mm."""
from typing import Any, Dict

REQUIRED_SHAPE_KEYS = ("M", "N", "K")


def validate_shape(shape: Dict[str, Any]) -> None:
    missing = [k for k in REQUIRED_SHAPE_KEYS if k not in shape]
    if missing:
        raise ValueError(f"Missing shape parameter(s): {', '.join(missing)}")
    for k in REQUIRED_SHAPE_KEYS:
        if int(shape[k]) <= 0:
            raise ValueError(f"{k} must be positive.")
    if int(shape["K"]) % 16:
        raise ValueError("K must be a multiple of 16.")
