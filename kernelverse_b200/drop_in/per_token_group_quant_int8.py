# ModelNew for operators/quantization/per_token_group_quant_int8 (B200 kernels).
import torch.nn as nn

from kernelverse_b200 import ops


class ModelNew(nn.Module):
    def __init__(self, shape):
        super().__init__()
        self.group_size = int(shape["group_size"])
        self.eps = float(shape["eps"])

    def forward(self, input_tensor):
        return ops.per_token_group_quant_int8(input_tensor, self.group_size, self.eps)
