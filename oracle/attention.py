"""CPU oracle for GQA decode attention over a paged cache (test infrastructure only).

Cache layout.  ``operators/attention/paged_attention_v1/paged_attention_v1.py:64-69``
gathers ``key_cache[block_table[b]]`` (declared ``[blocks, Hkv, bs, D]``) and then
``reshape(-1, Hkv, D)``; on a contiguous tensor that reshape reads each block's
memory as ``[bs, Hkv, D]``.  So token ``t`` of sequence ``b``, head ``h``, lives
in physical block ``block_table[b, t // bs]`` at row ``t % bs`` of a
``[bs, Hkv, D]`` block -- the same layout ``paged_kv_cache_update`` writes.
The oracle, like the device kernels, takes caches as ``[num_blocks, bs, Hkv, D]``.

* ``paged_attention_v1``: ``paged_attention_v1.py:27-92`` (q-head h reads KV
  head ``h // (Hq / Hkv)``; logits ``(K q) * scale``; float32 softmax).
* ``paged_attention_v2``: ``paged_attention_v2.py:28-175``; per partition of
  ``partition_size`` tokens: ``max_logits``, ``exp_sums``,
  ``tmp_out = weighted / (exp_sum + 1e-6)`` (``:158``) and the merged output
  ``/ (global_sum + 1e-6)`` (``:173``); partitions past a sequence's end keep
  ``exp_sum = 0``, ``max_logit = -inf``, ``tmp_out = 0``.
* ``batched_decode_attention``: ``operators/attention/batched_decode_attention/batched_decode_attention.py:30-52``
  over a dense ``[B, L, Hkv, D]`` cache with a ``pos < seq_len`` mask.
* ``paged_fp8_decode``: the BASELINE fourth config: the cache holds e4m3fn
  codes with per-KV-head float32 scales; values are ``code * scale[h]``.
* ``flash_attn_with_kvcache``: ``operators/attention/flash_attn_with_kvcache/flash_attn_with_kvcache.py:29-56``
  -- every query token of sequence b attends to its first ``cache_seqlens[b]`` keys of a
  dense ``[B, Sk, H, D]`` cache; also the natural-log sum of exp of the scaled logits.
* ``batched_prefill_attention``: ``operators/attention/batched_prefill_attention/batched_prefill_attention.py:30-73``
  -- packed requests delimited by ``qo_indptr`` / ``kv_indptr``; query row i of a request with
  ``q_len <= kv_len`` sits at position ``kv_len - q_len + i`` and sees keys ``<=`` it (``:66-73``).
* ``flash_decoding_attention``: ``operators/attention/flash_decoding_attention/flash_decoding_attention.py:30-87``
  over ``[B, H, S, D]`` caches in chunks of ``chunk_size`` keys, with the causal mask of
  ``:89-101`` (query i of Sq sees keys ``<= S - Sq + i``).

Everything is evaluated in float64 and returned as float32.
"""
from __future__ import annotations

import numpy as np

from .numerics import e4m3_decode


def gather_sequence(cache: np.ndarray, block_row: np.ndarray, seq_len: int) -> np.ndarray:
    """Tokens ``[seq_len, Hkv, D]`` of one sequence from a ``[nb, bs, Hkv, D]`` cache."""
    bs = cache.shape[1]
    nblk = (seq_len + bs - 1) // bs
    blocks = cache[np.asarray(block_row[:nblk], np.int64)]
    return blocks.reshape(-1, cache.shape[2], cache.shape[3])[:seq_len]


def _attend(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float):
    """q [D], k/v [L, D] (float64) -> (out, logits)."""
    logits = (k @ q) * scale
    m = logits.max()
    p = np.exp(logits - m)
    return (p @ v) / p.sum(), logits


def paged_attention_v1(query, key_cache, value_cache, seq_lens, block_table, scale: float) -> np.ndarray:
    q = np.asarray(query, np.float64)
    b_, hq, d = q.shape
    hkv = key_cache.shape[2]
    grp = hq // hkv
    out = np.zeros((b_, hq, d), np.float64)
    for b in range(b_):
        L = int(seq_lens[b])
        k = gather_sequence(np.asarray(key_cache, np.float64), block_table[b], L)
        v = gather_sequence(np.asarray(value_cache, np.float64), block_table[b], L)
        for h in range(hq):
            out[b, h], _ = _attend(q[b, h], k[:, h // grp], v[:, h // grp], scale)
    return out.astype(np.float32)


def paged_attention_v2(query, key_cache, value_cache, seq_lens, block_table, scale: float,
                       partition_size: int):
    q = np.asarray(query, np.float64)
    b_, hq, d = q.shape
    hkv = key_cache.shape[2]
    grp = hq // hkv
    max_len = int(np.max(seq_lens))
    P = (max_len + partition_size - 1) // partition_size
    out = np.zeros((b_, hq, d))
    exp_sums = np.zeros((b_, hq, P))
    max_logits = np.full((b_, hq, P), -np.inf)
    tmp_out = np.zeros((b_, hq, P, d))
    for b in range(b_):
        L = int(seq_lens[b])
        k = gather_sequence(np.asarray(key_cache, np.float64), block_table[b], L)
        v = gather_sequence(np.asarray(value_cache, np.float64), block_table[b], L)
        nparts = (L + partition_size - 1) // partition_size
        for h in range(hq):
            kk, vv = k[:, h // grp], v[:, h // grp]
            ws, ss, ms = [], [], []
            for p in range(nparts):
                lo, hi = p * partition_size, min((p + 1) * partition_size, L)
                logits = (kk[lo:hi] @ q[b, h]) * scale
                m = logits.max()
                e = np.exp(logits - m)
                s = e.sum()
                w = e @ vv[lo:hi]
                max_logits[b, h, p], exp_sums[b, h, p] = m, s
                tmp_out[b, h, p] = w / (s + 1e-6)
                ws.append(w); ss.append(s); ms.append(m)
            gm = max(ms)
            gs = sum(s * np.exp(m - gm) for s, m in zip(ss, ms))
            merged = sum(w * np.exp(m - gm) for w, m in zip(ws, ms))
            out[b, h] = merged / (gs + 1e-6)
    f = np.float32
    return out.astype(f), exp_sums.astype(f), max_logits.astype(f), tmp_out.astype(f)


def batched_decode_attention(q, k_cache, v_cache, seq_lens, scale: float) -> np.ndarray:
    q = np.asarray(q, np.float64)
    b_, hq, d = q.shape
    hkv = k_cache.shape[2]
    grp = hq // hkv
    out = np.zeros((b_, hq, d))
    for b in range(b_):
        L = int(seq_lens[b])
        for h in range(hq):
            k = np.asarray(k_cache[b, :L, h // grp], np.float64)
            v = np.asarray(v_cache[b, :L, h // grp], np.float64)
            out[b, h], _ = _attend(q[b, h], k, v, scale)
    return out.astype(np.float32)


def paged_fp8_decode(query, k_codes, v_codes, k_scale, v_scale, seq_lens, block_table, scale: float) -> np.ndarray:
    """Decode over an e4m3 cache; dequantises one sequence at a time to bound memory."""
    q = np.asarray(query, np.float64)
    b_, hq, d = q.shape
    hkv = k_codes.shape[2]
    grp = hq // hkv
    ks = np.asarray(k_scale, np.float64)
    vs = np.asarray(v_scale, np.float64)
    out = np.zeros((b_, hq, d))
    for b in range(b_):
        L = int(seq_lens[b])
        k = gather_sequence(k_codes, block_table[b], L)
        v = gather_sequence(v_codes, block_table[b], L)
        k = e4m3_decode(k).astype(np.float64) * ks[None, :, None]
        v = e4m3_decode(v).astype(np.float64) * vs[None, :, None]
        for h in range(hq):
            out[b, h], _ = _attend(q[b, h], k[:, h // grp], v[:, h // grp], scale)
    return out.astype(np.float32)


def flash_decoding_attention(query, key_cache, value_cache, chunk_size: int, causal: bool, scale: float):
    """Returns ``(output [B,H,Sq,D], exp_sums [B,H,Sq,P], max_logits [B,H,Sq,P], partial
    outputs [B,H,Sq,P,D])``.  Per chunk: ``max`` of the scaled scores (-inf when the chunk is
    fully masked), ``exp_sum`` of ``exp(score - max)`` (0 when masked), ``partial = weighted /
    max(exp_sum, 1e-6)``; merged as ``sum(partial * w) / max(sum(w), 1e-6)`` with
    ``w = exp_sum * exp(max - global_max)`` (flash_decoding_attention.py:46-87)."""
    q = np.asarray(query, np.float64)
    k = np.asarray(key_cache, np.float64)
    v = np.asarray(value_cache, np.float64)
    b_, h_, sq, d = q.shape
    s_ = k.shape[2]
    nch = (s_ + chunk_size - 1) // chunk_size
    es = np.zeros((b_, h_, sq, nch))
    mx = np.full((b_, h_, sq, nch), -np.inf)
    po = np.zeros((b_, h_, sq, nch, d))
    out = np.zeros((b_, h_, sq, d))
    for b in range(b_):
        for h in range(h_):
            for i in range(sq):
                limit = s_ - sq + i if causal else s_ - 1        # last visible key
                for c in range(nch):
                    k0, k1 = c * chunk_size, min((c + 1) * chunk_size, s_)
                    k1v = min(k1, limit + 1)
                    if k1v <= k0:
                        continue
                    sc = (k[b, h, k0:k1v] @ q[b, h, i]) * scale
                    m = sc.max()
                    p = np.exp(sc - m)
                    mx[b, h, i, c] = m
                    es[b, h, i, c] = p.sum()
                    po[b, h, i, c] = (p @ v[b, h, k0:k1v]) / max(p.sum(), 1e-6)
                gm = mx[b, h, i].max()
                w = es[b, h, i] * np.exp(mx[b, h, i] - gm)
                out[b, h, i] = (po[b, h, i] * w[:, None]).sum(0) / max(w.sum(), 1e-6)
    f = np.float32
    return out.astype(f), es.astype(f), mx.astype(f), po.astype(f)


def flash_attn_with_kvcache(q, k_cache, v_cache, cache_seqlens, scale: float):
    """Returns ``(output [B, Sq, H, D], softmax_lse [B, H, Sq])`` (flash_attn_with_kvcache.py:40-56);
    query head h reads KV head ``h // (H / Hkv)``."""
    qf = np.asarray(q, np.float64)
    k = np.asarray(k_cache, np.float64)
    v = np.asarray(v_cache, np.float64)
    b_, sq, h_, d = qf.shape
    grp = h_ // k.shape[2]
    out = np.zeros((b_, sq, h_, d))
    lse = np.zeros((b_, h_, sq))
    for b in range(b_):
        L = int(cache_seqlens[b])
        for h in range(h_):
            kk, vv = k[b, :L, h // grp], v[b, :L, h // grp]
            for i in range(sq):
                sc = (kk @ qf[b, i, h]) * scale
                m = sc.max()
                p = np.exp(sc - m)
                out[b, i, h] = (p @ vv) / p.sum()
                lse[b, h, i] = m + np.log(p.sum())
    return out.astype(np.float32), lse.astype(np.float32)



def batched_prefill_attention(q, k, v, qo_indptr, kv_indptr, num_q_heads: int, num_kv_heads: int, scale: float):
    """Packed causal prefill (batched_prefill_attention.py:30-73): ``q [Tq, Hq, D]``,
    ``k / v [Tkv, Hkv, D]``, indptrs ``[B + 1]`` -> ``out [Tq, Hq, D]``; query head h reads KV
    head ``h // (Hq / Hkv)``; row i of request b is at ``kv_len - q_len + i`` (:66-73)."""
    qf = np.asarray(q, np.float64)
    kf = np.asarray(k, np.float64)
    vf = np.asarray(v, np.float64)
    grp = num_q_heads // num_kv_heads
    out = np.zeros(qf.shape)
    qo = np.asarray(qo_indptr, np.int64)
    kvp = np.asarray(kv_indptr, np.int64)
    for b in range(len(qo) - 1):
        q0, q1, k0, k1 = qo[b], qo[b + 1], kvp[b], kvp[b + 1]
        ql, kl = q1 - q0, k1 - k0
        pos = np.arange(ql) + (kl - ql)
        masked = np.arange(kl)[None, :] > pos[:, None]
        for h in range(num_q_heads):
            kk, vv = kf[k0:k1, h // grp], vf[k0:k1, h // grp]
            sc = (qf[q0:q1, h] @ kk.T) * scale
            sc[masked] = -np.inf
            m = sc.max(axis=1, keepdims=True)
            p = np.exp(sc - m)
            out[q0:q1, h] = (p @ vv) / p.sum(axis=1, keepdims=True)
    return out.astype(np.float32)
