# ModelNew for operators/attention/flash_attn_with_kvcache (B200 kernels).
import torch.nn as nn

from kernelverse_b200 import ops


class ModelNew(nn.Module):
    def __init__(self, shape):
        super().__init__()
        self.scale = float(shape.get("softmax_scale", int(shape["head_dim"]) ** -0.5))

    def forward(self, q, k_cache, v_cache, cache_seqlens):
        return ops.flash_attn_with_kvcache(q, k_cache, v_cache, cache_seqlens, self.scale)
