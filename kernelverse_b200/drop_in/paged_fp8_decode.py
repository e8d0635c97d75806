# ModelNew for paged_fp8_decode (B200 kernels).
import torch.nn as nn

from kernelverse_b200 import ops


class ModelNew(nn.Module):
    def __init__(self, shape):
        super().__init__()
        self.scale = float(shape.get("softmax_scale", int(shape["head_dim"]) ** -0.5))

    def forward(self, query, k_cache, v_cache, k_scale, v_scale, seq_lens, block_table, k_new, v_new):
        return ops.paged_fp8_decode(query, k_cache, v_cache, k_scale, v_scale, seq_lens, block_table, self.scale,
                                    k_new=k_new, v_new=v_new)
