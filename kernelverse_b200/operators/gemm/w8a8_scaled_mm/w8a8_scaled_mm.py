"""W8A8 int8 GEMM with a per-token x per-channel scale epilogue (BASELINE third config).

acc = a[M, K] . b[N, K]^T accumulated exactly in int32; out = bf16((float32(acc) * a_scales[m]) * b_scales[n] + bias[n]).
Inputs: a, b int8 uniform in [-127, 127]; scales U(1e-3, 1e-2) float32; bias bf16 N(0, 0.1).
"""
from typing import Any, Dict, Tuple

import torch
import torch.nn as nn

from kernelverse_b200.operators.gemm.w8a8_scaled_mm.helpers import validate_shape


def _int_matmul(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    # float64 products of int8 values are exact and every partial sum stays below 2**53
    return (a.double() @ b.double().t()).to(torch.int64).to(torch.int32)


class Model(nn.Module):
    def __init__(self, shape: Dict[str, Any]) -> None:
        super().__init__()
        validate_shape(shape)

    def forward(self, a, b, a_scales, b_scales, bias) -> torch.Tensor:
        acc = _int_matmul(a, b)
        out = (acc.float() * a_scales.float()[:, None]) * b_scales.float()[None, :] + bias.float()[None, :]
        return out.to(torch.bfloat16)


def generate_inputs(shape: Dict[str, Any]) -> Tuple[torch.Tensor, ...]:
    validate_shape(shape)
    m, n, k = int(shape["M"]), int(shape["N"]), int(shape["K"])
    a = torch.randint(-127, 128, (m, k), dtype=torch.int8)
    b = torch.randint(-127, 128, (n, k), dtype=torch.int8)
    a_scales = torch.rand((m,), dtype=torch.float32) * 9e-3 + 1e-3
    b_scales = torch.rand((n,), dtype=torch.float32) * 9e-3 + 1e-3
    bias = (0.1 * torch.randn((n,), dtype=torch.float32)).to(torch.bfloat16)
    return a, b, a_scales, b_scales, bias
