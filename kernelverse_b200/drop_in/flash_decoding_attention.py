# ModelNew for operators/attention/flash_decoding_attention (B200 kernels).
import torch.nn as nn

from kernelverse_b200 import ops


class ModelNew(nn.Module):
    def __init__(self, shape):
        super().__init__()
        self.chunk_size = int(shape["chunk_size"])
        self.causal = bool(shape.get("causal", False))
        self.scale = float(shape.get("softmax_scale", int(shape["head_dim"]) ** -0.5))

    def forward(self, query, key_cache, value_cache):
        return ops.flash_decoding_attention(query, key_cache, value_cache, self.chunk_size, self.causal, self.scale)
