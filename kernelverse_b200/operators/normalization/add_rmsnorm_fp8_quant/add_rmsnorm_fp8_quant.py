"""Fused residual add + RMSNorm + per-token FP8 (e4m3) quantisation (BASELINE second config).

s = x + residual (float32); y = (s * rsqrt(mean(s^2) + eps)) * weight (float32, as add_rmsnorm's
correctness mode); scale = max(amax(|y|) / 448, 1/(448*512)); codes = e4m3(clamp(y / scale, +-448)).
Returns (residual_out = dtype(s), codes, scales float32 [rows]); ``codes`` are the e4m3fn bit
patterns as uint8.  KernelVerse's comparator (runner/generated_correctness_runner.py:414-423)
calls torch.isfinite on floating outputs, which CPU torch does not implement for float8 types,
so the package hands the codes over as bytes: its integer rule ``max_abs_diff`` (config.json:
1) then admits exactly one e4m3 step between codes of the same sign.
"""
from typing import Any, Dict, Tuple

import torch
import torch.nn as nn

from kernelverse_b200.operators.normalization.add_rmsnorm_fp8_quant.helpers import (E4M3_MAX, MIN_SCALING_FACTOR,
                                                                                     _resolve_dtype, validate_shape)


class Model(nn.Module):
    def __init__(self, shape: Dict[str, Any]) -> None:
        super().__init__()
        validate_shape(shape)
        self.eps = float(shape["eps"])
        self.dtype = _resolve_dtype(shape["dtype"])

    def forward(self, x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor):
        s = x.float() + residual.float()
        y = s * torch.rsqrt(s.pow(2).mean(dim=-1, keepdim=True) + self.eps) * weight.float()
        scales = (y.abs().amax(dim=-1, keepdim=True) / E4M3_MAX).clamp_min(MIN_SCALING_FACTOR)
        codes = (y / scales).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn)
        return s.to(self.dtype), codes.view(torch.uint8), scales.squeeze(-1)


def generate_inputs(shape: Dict[str, Any]) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    validate_shape(shape)
    dims = tuple(int(d) for d in shape["shape"])
    dt = _resolve_dtype(shape["dtype"])
    x = torch.randn(dims, dtype=torch.float32).to(dt)
    r = torch.randn(dims, dtype=torch.float32).to(dt)
    w = (1.0 + 0.02 * torch.randn((dims[-1],), dtype=torch.float32)).to(dt)
    return x, r, w
