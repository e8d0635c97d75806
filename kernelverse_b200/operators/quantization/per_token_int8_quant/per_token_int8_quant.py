"""Dynamic per-token symmetric int8 quantisation (BASELINE first config).

scale[t] = max(float32 amax(|x[t]|) / 127, 1e-6); q = clamp(round_half_even(x / scale), -127, 127).
Inputs: N(0, 1) with 0.1 % of the entries (seeded positions) multiplied by 50.
"""
from typing import Any, Dict, Tuple

import torch
import torch.nn as nn

from kernelverse_b200.operators.quantization.per_token_int8_quant.helpers import (EPS, INT8_QMAX, _resolve_dtype,
                                                                                   validate_shape)


class Model(nn.Module):
    def __init__(self, shape: Dict[str, Any]) -> None:
        super().__init__()
        validate_shape(shape)

    def forward(self, x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        xf = x.float()
        scales = (xf.abs().amax(dim=-1, keepdim=True) / INT8_QMAX).clamp_min(EPS)
        q = torch.round(xf / scales).clamp(-INT8_QMAX, INT8_QMAX).to(torch.int8)
        return q, scales.reshape(-1)


def generate_inputs(shape: Dict[str, Any]) -> Tuple[torch.Tensor]:
    validate_shape(shape)
    t, h = int(shape["num_tokens"]), int(shape["hidden_dim"])
    x = torch.randn((t, h), dtype=torch.float32)
    idx = torch.randperm(t * h)[: max(1, (t * h) // 1000)]
    x.view(-1)[idx] *= 50.0
    return (x.to(_resolve_dtype(shape["dtype"])),)
