# ModelNew for operators/gemm/int8_scaled_mm_azp (B200 tensor-core kernels).
import torch
import torch.nn as nn

from kernelverse_b200 import ops

_DT = {"FP32": torch.float32, "FP16": torch.float16, "BF16": torch.bfloat16}


class ModelNew(nn.Module):
    def __init__(self, shape):
        super().__init__()
        self.has_azp = bool(shape["has_azp"])
        self.has_bias = bool(shape["has_bias"])
        self.output_dtype = _DT[shape["output_dtype"]]

    def forward(self, a, b, a_scales, b_scales, azp_adj, azp, bias):
        return ops.int8_scaled_mm_azp(a, b, a_scales, b_scales, azp_adj, azp, bias, self.has_azp, self.has_bias,
                                      self.output_dtype)
