# ModelNew for add_rmsnorm_fp8_quant (B200 kernels).
import torch
import torch.nn as nn

from kernelverse_b200 import ops


class ModelNew(nn.Module):
    def __init__(self, shape):
        super().__init__()
        self.eps = float(shape["eps"])

    def forward(self, x, residual, weight):
        residual_out, codes, scales = ops.add_rmsnorm_quant(x, residual, weight, self.eps)
        return residual_out, codes.view(torch.uint8), scales
