"""Paged FP8 KV-cache write + GQA decode attention (BASELINE fourth config).

Caches are [num_blocks, block_size, Hkv, D] float8_e4m3fn codes with one float32 scale per KV
head (the memory order KernelVerse's paged_attention_v1 reads and paged_kv_cache_update
writes).  The newest token of sequence b (position L_b - 1) is first written to slot
block_table[b][(L_b-1)//bs]*bs + (L_b-1)%bs as e4m3(clamp(new / scale[h], +-448)); then every
query head h attends over the L_b tokens of KV head h // (Hq / Hkv) with float32 softmax.
"""
from typing import Any, Dict, Tuple

import torch
import torch.nn as nn

from kernelverse_b200.operators.attention.paged_fp8_decode.helpers import E4M3_MAX, validate_shape


class Model(nn.Module):
    def __init__(self, shape: Dict[str, Any]) -> None:
        super().__init__()
        validate_shape(shape)
        self.scale = float(shape.get("softmax_scale", int(shape["head_dim"]) ** -0.5))

    def forward(self, query, k_cache, v_cache, k_scale, v_scale, seq_lens, block_table, k_new, v_new):
        bs = k_cache.shape[1]
        hkv = k_cache.shape[2]
        b_, hq, d = query.shape
        grp = hq // hkv
        ks = k_scale.float()[None, :, None]
        vs = v_scale.float()[None, :, None]
        out = torch.empty((b_, hq, d), dtype=torch.float32, device=query.device)
        kflat = k_cache.view(-1, hkv, d)
        vflat = v_cache.view(-1, hkv, d)
        for b in range(b_):
            L = int(seq_lens[b].item())
            slot = int(block_table[b, (L - 1) // bs].item()) * bs + (L - 1) % bs
            kflat[slot] = (k_new[b].float() / ks[0]).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn)
            vflat[slot] = (v_new[b].float() / vs[0]).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn)
            nblk = (L + bs - 1) // bs
            blocks = block_table[b, :nblk].long()
            k = k_cache[blocks].reshape(-1, hkv, d)[:L].float() * ks
            v = v_cache[blocks].reshape(-1, hkv, d)[:L].float() * vs
            for h in range(hq):
                logits = (k[:, h // grp] @ query[b, h].float()) * self.scale
                out[b, h] = torch.softmax(logits, dim=-1) @ v[:, h // grp]
        return out.to(query.dtype)


def generate_inputs(shape: Dict[str, Any]) -> Tuple[torch.Tensor, ...]:
    validate_shape(shape)
    b_, hq, hkv, d, bs = (int(shape[k]) for k in ("batch_size", "num_q_heads", "num_kv_heads", "head_dim", "block_size"))
    lens = torch.randint(int(shape["min_context"]), int(shape["max_context"]) + 1, (b_,), dtype=torch.int32)
    nblk = (lens + bs - 1) // bs
    total = int(nblk.sum())
    perm = torch.randperm(total).to(torch.int32)
    table = torch.zeros((b_, int(nblk.max())), dtype=torch.int32)   # unused entries point at block 0
    pos = 0
    for b in range(b_):
        n = int(nblk[b])
        table[b, :n] = perm[pos:pos + n]
        pos += n
    k_scale = torch.rand((hkv,), dtype=torch.float32) * 0.01 + 0.005
    v_scale = torch.rand((hkv,), dtype=torch.float32) * 0.01 + 0.005
    k_cache = (torch.randn((total, bs, hkv, d)) / k_scale[None, None, :, None]).clamp(-E4M3_MAX, E4M3_MAX).to(
        torch.float8_e4m3fn)
    v_cache = (torch.randn((total, bs, hkv, d)) / v_scale[None, None, :, None]).clamp(-E4M3_MAX, E4M3_MAX).to(
        torch.float8_e4m3fn)
    query = torch.randn((b_, hq, d)).to(torch.bfloat16)
    k_new = torch.randn((b_, hkv, d)).to(torch.bfloat16)
    v_new = torch.randn((b_, hkv, d)).to(torch.bfloat16)
    return query, k_cache, v_cache, k_scale, v_scale, lens, table, k_new, v_new
