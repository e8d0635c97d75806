# ModelNew for operators/kv_cache/paged_kv_cache_update (B200 kernels).
import torch.nn as nn

from kernelverse_b200 import ops


class ModelNew(nn.Module):
    def __init__(self, shape):
        super().__init__()

    def forward(self, to_cache, kv_cache, slot_mapping):
        return ops.paged_kv_cache_update(to_cache, kv_cache, slot_mapping)
