# ModelNew for operators/attention/batched_decode_attention (B200 kernels).
import torch
import torch.nn as nn

from kernelverse_b200 import ops

_DT = {"FP32": torch.float32, "FP16": torch.float16, "BF16": torch.bfloat16}


class ModelNew(nn.Module):
    def __init__(self, shape):
        super().__init__()
        self.scale = float(shape.get("softmax_scale", int(shape["head_dim"]) ** -0.5))
        self.output_dtype = _DT[shape["dtype"]]

    def forward(self, q, k_cache, v_cache, seq_lens):
        return ops.batched_decode_attention(q, k_cache, v_cache, seq_lens, self.scale, self.output_dtype)
