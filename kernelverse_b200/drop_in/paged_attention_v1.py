# ModelNew for operators/attention/paged_attention_v1 (B200 kernels).
import torch
import torch.nn as nn

from kernelverse_b200 import ops

_DT = {"FP32": torch.float32, "FP16": torch.float16, "BF16": torch.bfloat16}


class ModelNew(nn.Module):
    def __init__(self, shape):
        super().__init__()
        self.scale = float(shape.get("softmax_scale", int(shape["head_dim"]) ** -0.5))
        self.output_dtype = _DT[str(shape["output_dtype"])]

    def forward(self, query, key_cache, value_cache, seq_lens, block_table):
        return ops.paged_attention_v1(query, key_cache, value_cache, seq_lens, block_table, self.scale,
                                      self.output_dtype)
