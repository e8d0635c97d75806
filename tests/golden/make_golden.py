"""Generate the golden fixtures in this directory by running the REFERENCE on CPU.

Run once, in a container where the KernelVerse reference is importable::

    KV_REFERENCE_ROOT=<path to KernelVerse checkout> python tests/golden/make_golden.py

``KV_GOLDEN_ONLY=prefix1,prefix2`` writes only the fixtures whose names start with one of
the prefixes (the others are computed but left untouched).

Each fixture is a small ``.npz`` holding the seeded inputs (made by the
reference's own ``generate_inputs`` where one exists) and the outputs of the
reference's ``Model.forward`` on CPU.  bf16 tensors are stored as uint16 bit
patterns and float8_e4m3fn tensors as uint8 codes; ``<name>__dtype`` records
the torch dtype.  The fixtures pin the numpy oracle (``tests/test_oracle_golden.py``)
and the device kernels (``tests/test_gpu_*.py``); nothing at test or bench
time reads the reference itself.

The BASELINE variants that have no reference operator (fused add+RMSNorm+FP8,
the W8A8 epilogue with an int32 accumulator, the FP8 paged cache) are produced
by composing the reference operators with PyTorch's own primitives
(``torch._int_mm``, the ``float8_e4m3fn`` cast), as noted per fixture.
"""
from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REF = os.environ.get("KV_REFERENCE_ROOT")
if not REF or not Path(REF, "operators", "registry.py").exists():
    sys.exit("set KV_REFERENCE_ROOT to a KernelVerse checkout")
sys.path.insert(0, REF)
sys.dont_write_bytecode = True

from operators.registry import load_object  # noqa: E402

MIN_SCALING_FACTOR = 1.0 / (448.0 * 512.0)


def _op(category: str, name: str, attr: str):
    return load_object(f"{REF}/operators/{category}/{name}/{name}.py::{attr}")


def _np(t: torch.Tensor):
    t = t.detach().contiguous().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    if t.dtype == torch.float8_e4m3fn:
        return t.view(torch.uint8).numpy()
    return t.numpy()


ONLY = [p for p in os.environ.get("KV_GOLDEN_ONLY", "").split(",") if p]


def save(name: str, meta: dict, **tensors):
    if ONLY and not any(name.startswith(p) for p in ONLY):   # regenerate a subset only
        return
    arrays = {}
    for k, v in tensors.items():
        if isinstance(v, torch.Tensor):
            arrays[k] = _np(v)
            arrays[k + "__dtype"] = np.array(str(v.dtype).replace("torch.", ""))
        else:
            arrays[k] = np.asarray(v)
    arrays["meta"] = np.array(json.dumps(meta))
    np.savez_compressed(HERE / f"{name}.npz", **arrays)
    print("wrote", name, {k: tuple(v.shape) for k, v in arrays.items() if not k.endswith("__dtype") and k != "meta"})


def run_model(category, name, shape, inputs, mode="correctness"):
    shape = dict(shape, _baseline_compute_mode=mode)
    model = _op(category, name, "Model")(shape).eval()
    with torch.no_grad():
        return model(*inputs)


def gen_inputs(category, name, shape, seed):
    torch.manual_seed(seed)
    return _op(category, name, "generate_inputs")(shape)


def main():
    torch.set_num_threads(1)
    # --- a1: dynamic_scaled_int8_quant (per-tensor), all three input dtypes + 1-D + 3-D
    for i, (dims, dt) in enumerate([([16, 64], "FP32"), ([16, 64], "FP16"), ([16, 64], "BF16"),
                                    ([2, 8, 32], "BF16"), ([300], "FP32"), ([3, 37], "FP16")]):
        shape = {"dims": dims, "dtype": dt}
        (x,) = gen_inputs("quantization", "dynamic_scaled_int8_quant", shape, 100 + i)
        q, s, azp = run_model("quantization", "dynamic_scaled_int8_quant", shape, (x,))
        save(f"dynamic_scaled_int8_quant_{i}", shape, x=x, q=q, scale=s, azp=azp)

    # --- a2: per_token_group_quant_int8, incl. group == hidden (per-token, BASELINE first config form)
    for i, (t, h, g, dt) in enumerate([(32, 256, 64, "FP32"), (32, 256, 64, "BF16"), (17, 128, 32, "FP16"),
                                      (24, 512, 512, "BF16"), (8, 96, 96, "FP32")]):
        shape = {"num_tokens": t, "hidden_dim": h, "group_size": g, "dtype": dt, "eps": 1e-6}
        (x,) = gen_inputs("quantization", "per_token_group_quant_int8", shape, 200 + i)
        if i == 3:  # BASELINE first config distribution: N(0,1) with 0.1% of entries x50, and one all-zero row
            gen = torch.Generator().manual_seed(201)
            xf = torch.randn(x.shape, generator=gen)
            idx = torch.randperm(xf.numel(), generator=gen)[: max(1, xf.numel() // 1000)]
            xf.view(-1)[idx] *= 50.0
            xf[5] = 0.0
            x = xf.to(x.dtype)
        q, s = run_model("quantization", "per_token_group_quant_int8", shape, (x,))
        save(f"per_token_group_quant_int8_{i}", shape, x=x, q=q, scales=s)

    # --- a3: add_rmsnorm (reference op), correctness mode, three dtypes incl. 3-D
    for i, (shp, dt) in enumerate([([4, 256], "FP32"), ([4, 256], "BF16"), ([3, 5, 64], "FP16"), ([2, 1000], "BF16")]):
        shape = {"shape": shp, "eps": 1e-6, "dtype": dt}
        x, r, w = gen_inputs("normalization", "add_rmsnorm", shape, 300 + i)
        if i == 1:
            w = (1.0 + 0.02 * torch.randn(w.shape, generator=torch.Generator().manual_seed(3))).to(w.dtype)
        y = run_model("normalization", "add_rmsnorm", shape, (x, r, w))
        save(f"add_rmsnorm_{i}", shape, x=x, residual=r, weight=w, out=y)

    # --- a3+a4: fused add + RMSNorm + per-row e4m3 quant (BASELINE second config form), composed from
    #     the reference add_rmsnorm (correctness mode, FP32 output) and torch's float8_e4m3fn cast.
    for i, (m, h) in enumerate([(8, 256), (3, 1024)]):
        gen = torch.Generator().manual_seed(400 + i)
        x = torch.randn((m, h), generator=gen).to(torch.bfloat16)
        r = torch.randn((m, h), generator=gen).to(torch.bfloat16)
        w = (1.0 + 0.02 * torch.randn((h,), generator=gen)).to(torch.bfloat16)
        y = run_model("normalization", "add_rmsnorm", {"shape": [m, h], "eps": 1e-6, "dtype": "FP32"}, (x, r, w))
        r_out = (x.float() + r.float()).to(torch.bfloat16)
        scale = (y.abs().amax(dim=-1, keepdim=True) / 448.0).clamp_min(MIN_SCALING_FACTOR)
        codes = (y / scale).clamp(-448.0, 448.0).to(torch.float8_e4m3fn)
        save(f"add_rmsnorm_fp8_{i}", {"M": m, "H": h, "eps": 1e-6}, x=x, residual=r, weight=w,
             y=y, residual_out=r_out, codes=codes, scales=scale.reshape(-1))

    # --- a5: int8_scaled_mm_azp (reference op, B is [K, N])
    for i, (m, n, k, azp, bias, dt) in enumerate([(8, 32, 64, True, True, "FP32"), (5, 48, 96, False, True, "BF16"),
                                                  (16, 16, 128, True, False, "FP16"), (1, 24, 32, False, False, "FP32")]):
        shape = {"M": m, "N": n, "K": k, "has_azp": azp, "has_bias": bias, "output_dtype": dt}
        ins = gen_inputs("gemm", "int8_scaled_mm_azp", shape, 500 + i)
        out = run_model("gemm", "int8_scaled_mm_azp", shape, ins)
        names = ["a", "b", "a_scales", "b_scales", "azp_adj", "azp", "bias"]
        save(f"int8_scaled_mm_azp_{i}", shape, out=out, **dict(zip(names, ins)))

    # --- a5: W8A8 (BASELINE third config form): int32 acc via torch._int_mm, float32 epilogue, bf16 out
    for i, (m, n, k) in enumerate([(16, 64, 128), (33, 40, 256)]):
        gen = torch.Generator().manual_seed(600 + i)
        a = torch.randint(-127, 128, (m, k), generator=gen, dtype=torch.int8)
        b = torch.randint(-127, 128, (n, k), generator=gen, dtype=torch.int8)
        sa = torch.rand((m,), generator=gen) * 9e-3 + 1e-3
        sb = torch.rand((n,), generator=gen) * 9e-3 + 1e-3
        bias = (0.1 * torch.randn((n,), generator=gen)).to(torch.bfloat16)
        mp = max(m, 17)  # torch._int_mm wants m > 16
        ap = torch.zeros((mp, k), dtype=torch.int8)
        ap[:m] = a
        acc = torch._int_mm(ap, b.t().contiguous())[:m]
        out = ((acc.float() * sa[:, None]) * sb[None, :] + bias.float()[None, :]).to(torch.bfloat16)
        save(f"w8a8_{i}", {"M": m, "N": n, "K": k}, a=a, b=b, sa=sa, sb=sb, bias=bias, acc=acc, out=out)

    # --- a6: paged_kv_cache_update (reference op), with and without invalid slots, both index dtypes
    for i, (t, nb, bs, h, d, dt, idt, inv) in enumerate([(16, 8, 4, 2, 16, "FP32", "INT64", True),
                                                        (20, 6, 8, 2, 32, "BF16", "INT32", False),
                                                        (9, 4, 16, 1, 64, "FP16", "INT64", True)]):
        shape = {"num_tokens": t, "num_blocks": nb, "block_size": bs, "num_heads": h, "head_dim": d,
                 "dtype": dt, "index_dtype": idt, "has_invalid_slots": inv}
        to_cache, kv_cache, slots = gen_inputs("kv_cache", "paged_kv_cache_update", shape, 700 + i)
        kv_cache = torch.randn(kv_cache.shape, generator=torch.Generator().manual_seed(7)).to(kv_cache.dtype)
        out = run_model("kv_cache", "paged_kv_cache_update", shape, (to_cache, kv_cache, slots))
        save(f"paged_kv_cache_update_{i}", shape, to_cache=to_cache, kv_cache=kv_cache, slot_mapping=slots, out=out)

    # --- a7/a8: paged attention v1 / v2 (reference ops) on ragged lengths and a permuted block table.
    for i, (b, lens, hq, hkv, d, bs, part, dt) in enumerate([
            (3, [40, 17, 64], 4, 2, 16, 16, 16, "FP32"),
            (2, [33, 5], 8, 1, 32, 8, 32, "BF16"),
            (4, [64, 64, 1, 50], 4, 4, 64, 16, 64, "FP16")]):
        gen = torch.Generator().manual_seed(800 + i)
        tdt = {"FP32": torch.float32, "BF16": torch.bfloat16, "FP16": torch.float16}[dt]
        maxb = (max(lens) + bs - 1) // bs
        nblocks = b * maxb + 3
        q = torch.randn((b, hq, d), generator=gen).to(tdt)
        kc = torch.randn((nblocks, bs, hkv, d), generator=gen).to(tdt)   # memory layout [nb, bs, Hkv, D]
        vc = torch.randn((nblocks, bs, hkv, d), generator=gen).to(tdt)
        perm = torch.randperm(nblocks, generator=gen)[: b * maxb].to(torch.int32)
        bt = perm.view(b, maxb).contiguous()
        for j, L in enumerate(lens):  # pad unused entries with a valid block index (0)
            bt[j, (L + bs - 1) // bs:] = 0
        sl = torch.tensor(lens, dtype=torch.int32)
        shape = {"batch_size": b, "seq_len": max(lens), "num_q_heads": hq, "num_kv_heads": hkv, "head_dim": d,
                 "block_size": bs, "input_dtype": dt, "output_dtype": dt, "partition_size": part}
        # the reference declares [nb, Hkv, bs, D]; pass the same memory viewed that way
        kd, vd = kc.view(nblocks, hkv, bs, d), vc.view(nblocks, hkv, bs, d)
        out1 = run_model("attention", "paged_attention_v1", shape, (q, kd, vd, sl, bt))
        out2 = run_model("attention", "paged_attention_v2", shape, (q, kd, vd, sl, bt))
        save(f"paged_attention_{i}", shape, query=q, key_cache=kc, value_cache=vc, seq_lens=sl, block_table=bt,
             out_v1=out1, out_v2=out2[0], exp_sums=out2[1], max_logits=out2[2], tmp_out=out2[3])

    # --- a9: batched_decode_attention (reference op), ragged
    for i, (b, L, hq, hkv, d, pat, dt) in enumerate([(3, 20, 4, 2, 16, "ragged", "FP32"),
                                                    (4, 33, 8, 8, 32, "highly_ragged", "BF16")]):
        shape = {"batch_size": b, "max_seq_len": L, "num_q_heads": hq, "num_kv_heads": hkv, "head_dim": d,
                 "seq_len_pattern": pat, "dtype": dt}
        ins = gen_inputs("attention", "batched_decode_attention", shape, 900 + i)
        out = run_model("attention", "batched_decode_attention", shape, ins)
        save(f"batched_decode_attention_{i}", shape, q=ins[0], k_cache=ins[1], v_cache=ins[2], seq_lens=ins[3], out=out)

    # --- a6+a7 FP8 (BASELINE fourth config form): e4m3 cache with per-head scales, new token written at
    #     slot bt[b][(L-1)//bs]*bs + (L-1)%bs, then v1 over the dequantised cache (correctness mode).
    for i, (b, lens, hq, hkv, d, bs) in enumerate([(3, [37, 16, 70], 8, 2, 64, 16), (2, [1, 48], 4, 1, 128, 16)]):
        gen = torch.Generator().manual_seed(1000 + i)
        maxb = (max(lens) + bs - 1) // bs
        nblocks = b * maxb + 2
        k_scale = torch.rand((hkv,), generator=gen) * 0.01 + 0.005
        v_scale = torch.rand((hkv,), generator=gen) * 0.01 + 0.005
        kc = (torch.randn((nblocks, bs, hkv, d), generator=gen) / k_scale[None, None, :, None]).clamp(-448, 448).to(torch.float8_e4m3fn)
        vc = (torch.randn((nblocks, bs, hkv, d), generator=gen) / v_scale[None, None, :, None]).clamp(-448, 448).to(torch.float8_e4m3fn)
        perm = torch.randperm(nblocks, generator=gen)[: b * maxb].to(torch.int32)
        bt = perm.view(b, maxb).contiguous()
        for j, L in enumerate(lens):
            bt[j, (L + bs - 1) // bs:] = 0
        sl = torch.tensor(lens, dtype=torch.int32)
        q = torch.randn((b, hq, d), generator=gen).to(torch.bfloat16)
        k_new = torch.randn((b, hkv, d), generator=gen).to(torch.bfloat16)
        v_new = torch.randn((b, hkv, d), generator=gen).to(torch.bfloat16)
        slots = torch.tensor([int(bt[j, (L - 1) // bs]) * bs + (L - 1) % bs for j, L in enumerate(lens)], dtype=torch.int64)
        kq = (k_new.float() / k_scale[None, :, None]).clamp(-448, 448).to(torch.float8_e4m3fn)
        vq = (v_new.float() / v_scale[None, :, None]).clamp(-448, 448).to(torch.float8_e4m3fn)
        shp_u = {"num_tokens": b, "num_blocks": nblocks, "block_size": bs, "num_heads": hkv, "head_dim": d,
                 "dtype": "FP32", "index_dtype": "INT64", "has_invalid_slots": False}
        # slot placement through the reference scatter (on the codes' byte patterns, viewed as uint8 -> float32)
        kc_after = run_model("kv_cache", "paged_kv_cache_update", shp_u,
                             (kq.view(torch.uint8).float(), kc.view(torch.uint8).float(), slots)).to(torch.uint8).view(torch.float8_e4m3fn)
        vc_after = run_model("kv_cache", "paged_kv_cache_update", shp_u,
                             (vq.view(torch.uint8).float(), vc.view(torch.uint8).float(), slots)).to(torch.uint8).view(torch.float8_e4m3fn)
        kd = (kc_after.float() * k_scale[None, None, :, None]).view(nblocks, hkv, bs, d)
        vd = (vc_after.float() * v_scale[None, None, :, None]).view(nblocks, hkv, bs, d)
        shape = {"batch_size": b, "seq_len": max(lens), "num_q_heads": hq, "num_kv_heads": hkv, "head_dim": d,
                 "block_size": bs, "input_dtype": "FP32", "output_dtype": "FP32"}
        out = run_model("attention", "paged_attention_v1", shape, (q.float(), kd, vd, sl, bt))
        save(f"paged_fp8_decode_{i}", shape, query=q, k_cache=kc, v_cache=vc, k_scale=k_scale, v_scale=v_scale,
             k_new=k_new, v_new=v_new, seq_lens=sl, block_table=bt, slot_mapping=slots,
             k_cache_after=kc_after, v_cache_after=vc_after, out=out)

    # --- next rows: static_scaled_int8_quant (reference op, correctness mode), incl. a zero point,
    #     a scale below MIN_SCALE and values that clamp
    for i, (dims, dt, sc, zp) in enumerate([([16, 64], "FP32", 0.125, 0), ([4, 96], "BF16", 0.05, 3),
                                            ([2, 8, 40], "FP16", 1e-9, -2), ([300], "FP32", 0.01, 0)]):
        shape = {"dims": dims, "dtype": dt}
        x, _, _ = gen_inputs("quantization", "static_scaled_int8_quant", shape, 1100 + i)
        if i == 3:
            x = x * 2.0                                            # a share of values beyond +-127 * scale
        scale = torch.tensor([sc], dtype=torch.float32)
        azp = torch.tensor([zp], dtype=torch.int32)
        q = run_model("quantization", "static_scaled_int8_quant", shape, (x, scale, azp))
        save(f"static_scaled_int8_quant_{i}", shape, x=x, scale=scale, azp=azp, q=q)

    # --- next rows: kv_cache_write (reference op, performance mode as its config.json sets), shared and
    #     per-batch positions
    for i, (b, h, smax, w, d, mode, dt) in enumerate([(2, 2, 32, 1, 16, "shared", "FP32"),
                                                     (3, 2, 40, 5, 32, "per_batch", "BF16"),
                                                     (2, 1, 24, 8, 80, "per_batch", "FP16")]):
        shape = {"batch_size": b, "num_kv_heads": h, "max_seq_len": smax, "write_seq_len": w, "head_dim": d,
                 "position_mode": mode, "dtype": dt}
        kc, vc, k, v, pos = gen_inputs("kv_cache", "kv_cache_write", shape, 1200 + i)
        ko, vo = run_model("kv_cache", "kv_cache_write", shape, (kc, vc, k, v, pos), mode="performance")
        save(f"kv_cache_write_{i}", shape, key_cache=kc, value_cache=vc, key=k, value=v, positions=pos,
             key_out=ko, value_out=vo)

    # --- next rows: flash_decoding_attention (reference op, correctness mode), single and multi query,
    #     causal and not
    for i, (b, sq, s, h, d, ch, causal, dt) in enumerate([(2, 1, 300, 2, 64, 64, False, "FP32"),
                                                        (1, 4, 200, 2, 128, 64, True, "BF16"),
                                                        (2, 3, 96, 3, 64, 32, False, "FP16"),
                                                        (1, 32, 64, 1, 64, 16, True, "FP32")]):
        shape = {"batch_size": b, "query_seq_len": sq, "kv_seq_len": s, "num_heads": h, "head_dim": d,
                 "chunk_size": ch, "causal": causal, "dtype": dt}
        qq, kk, vv = gen_inputs("attention", "flash_decoding_attention", shape, 1300 + i)
        out, es, ml, po = run_model("attention", "flash_decoding_attention", shape, (qq, kk, vv))
        save(f"flash_decoding_attention_{i}", shape, query=qq, key_cache=kk, value_cache=vv, out=out,
             exp_sums=es, max_logits=ml, partial_out=po)

    # --- next rows: W8A8 gate+up GEMM followed by the reference's swiglu / mul_and_silu (correctness mode)
    #     on the bf16 GEMM output (int32 acc via torch._int_mm, float32 epilogue as the w8a8 fixtures)
    for i, (m, inner, k, act) in enumerate([(33, 256, 256, "swiglu"), (200, 128, 128, "mul_and_silu")]):
        gen = torch.Generator().manual_seed(1400 + i)
        a = torch.randint(-127, 128, (m, k), generator=gen, dtype=torch.int8)
        b1 = torch.randint(-127, 128, (inner, k), generator=gen, dtype=torch.int8)
        b2 = torch.randint(-127, 128, (inner, k), generator=gen, dtype=torch.int8)
        sa = torch.rand((m,), generator=gen) * 9e-3 + 1e-3
        s1 = torch.rand((inner,), generator=gen) * 9e-3 + 1e-3
        s2 = torch.rand((inner,), generator=gen) * 9e-3 + 1e-3
        bias1 = (0.1 * torch.randn((inner,), generator=gen)).to(torch.bfloat16)
        bias2 = (0.1 * torch.randn((inner,), generator=gen)).to(torch.bfloat16)
        mp = max(m, 17)
        ap = torch.zeros((mp, k), dtype=torch.int8)
        ap[:m] = a
        y1 = ((torch._int_mm(ap, b1.t().contiguous())[:m].float() * sa[:, None]) * s1[None, :] + bias1.float()).to(torch.bfloat16)
        y2 = ((torch._int_mm(ap, b2.t().contiguous())[:m].float() * sa[:, None]) * s2[None, :] + bias2.float()).to(torch.bfloat16)
        x = torch.cat([y1, y2], dim=-1)
        shp = {"shape": [m, 2 * inner], "dim": -1, "dtype": "BF16"}
        out = run_model("activation", act, shp, (x,))
        save(f"w8a8_act_{i}", {"M": m, "I": inner, "K": k, "act": act}, a=a, b_first=b1, b_second=b2, sa=sa,
             s_first=s1, s_second=s2, bias_first=bias1, bias_second=bias2, out=out)

    # --- next rows: flash_attn_with_kvcache (reference op, correctness mode): ragged cache lengths,
    #     several query tokens, and 32 heads (split over CTAs on the device)
    for i, (b, sq, sk, h, d, pat, dt) in enumerate([(3, 1, 300, 4, 64, "ragged", "FP32"),
                                                   (3, 4, 200, 2, 128, "ragged", "BF16"),
                                                   (2, 8, 96, 32, 64, "full", "FP16"),
                                                   (4, 2, 130, 32, 128, "ragged", "BF16")]):
        shape = {"batch_size": b, "seq_len_q": sq, "seq_len_k": sk, "num_heads": h, "head_dim": d,
                 "cache_pattern": pat, "dtype": dt}
        qq, kk, vv, lens = gen_inputs("attention", "flash_attn_with_kvcache", shape, 1500 + i)
        out, lse = run_model("attention", "flash_attn_with_kvcache", shape, (qq, kk, vv, lens))
        save(f"flash_attn_with_kvcache_{i}", shape, q=qq, k_cache=kk, v_cache=vv, cache_seqlens=lens, out=out,
             softmax_lse=lse)

    # --- next rows: batched_prefill_attention (reference op, correctness mode): full and chunked
    #     prefill, ragged lengths, GQA / MHA / MQA, head dims 64 / 80 / 96 / 128, all three dtypes
    for i, (ql, kl, hq, hkv, d, dt) in enumerate([([64, 48, 32, 16], [64, 48, 32, 16], 8, 2, 64, "FP32"),
                                                 ([100, 7], [100, 7], 4, 4, 128, "BF16"),
                                                 ([33, 70], [160, 70], 8, 1, 80, "FP16"),
                                                 ([129, 1, 65], [200, 1, 65], 4, 2, 96, "FP32"),
                                                 ([80, 40], [300, 90], 8, 2, 128, "BF16")]):
        shape = {"q_lens": ql, "kv_lens": kl, "num_q_heads": hq, "num_kv_heads": hkv, "head_dim": d, "dtype": dt}
        qq, kk, vv, qo, kvp = gen_inputs("attention", "batched_prefill_attention", shape, 1600 + i)
        out = run_model("attention", "batched_prefill_attention", shape, (qq, kk, vv, qo, kvp))
        save(f"batched_prefill_attention_{i}", shape, q=qq, k=kk, v=vv, qo_indptr=qo, kv_indptr=kvp, out=out)

    (HERE / "VERSIONS.txt").write_text(f"torch {torch.__version__}\nnumpy {np.__version__}\n")


if __name__ == "__main__":
    main()
