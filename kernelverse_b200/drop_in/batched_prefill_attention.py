# ModelNew for operators/attention/batched_prefill_attention (B200 kernels).
import torch.nn as nn

from kernelverse_b200 import ops


class ModelNew(nn.Module):
    def __init__(self, shape):
        super().__init__()
        self.scale = float(shape.get("softmax_scale", int(shape["head_dim"]) ** -0.5))

    def forward(self, q, k, v, qo_indptr, kv_indptr):
        return ops.batched_prefill_attention(q, k, v, qo_indptr, kv_indptr, self.scale)
