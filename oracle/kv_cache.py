"""CPU oracle for paged KV-cache writes (test infrastructure only).

* ``paged_kv_cache_update`` restates
  ``operators/kv_cache/paged_kv_cache_update/paged_kv_cache_update.py:21-31``:
  the output is a copy of ``kv_cache`` ``[num_blocks, block_size, H, D]`` in
  which flat slot ``slot_mapping[i]`` (skipped when negative) receives token
  ``i`` of ``to_cache`` ``[T, H, D]``.
* ``paged_fp8_kv_write`` is the BASELINE fourth config's write: the same slot
  placement, into an e4m3fn cache of the same layout, with per-KV-head float32
  scales: ``code = e4m3(clamp(x / scale[h], -448, 448))``.
* ``decode_slots`` gives the slot of each sequence's newest token,
  ``block_table[b][(ctx_b - 1) // bs] * bs + (ctx_b - 1) % bs``.
"""
from __future__ import annotations

import numpy as np

from .numerics import e4m3_quantize


def paged_kv_cache_update(to_cache: np.ndarray, kv_cache: np.ndarray, slot_mapping: np.ndarray) -> np.ndarray:
    out = np.array(kv_cache, copy=True)
    flat = out.reshape(-1, *out.shape[2:])
    slots = np.asarray(slot_mapping).astype(np.int64)
    for i, s in enumerate(slots):
        if s >= 0:
            flat[s] = to_cache[i]
    return out


def decode_slots(seq_lens: np.ndarray, block_table: np.ndarray, block_size: int) -> np.ndarray:
    pos = np.asarray(seq_lens, np.int64) - 1
    blk = np.asarray(block_table, np.int64)[np.arange(len(pos)), pos // block_size]
    return blk * block_size + pos % block_size


def paged_fp8_kv_write(x_new: np.ndarray, cache_codes: np.ndarray, slot_mapping: np.ndarray,
                       head_scales: np.ndarray) -> np.ndarray:
    """Write ``x_new`` ``[T, Hkv, D]`` into the uint8 e4m3 cache ``[nb, bs, Hkv, D]``."""
    out = np.array(cache_codes, copy=True)
    flat = out.reshape(-1, *out.shape[2:])
    codes = e4m3_quantize(x_new, np.asarray(head_scales, np.float32)[None, :, None])
    for i, s in enumerate(np.asarray(slot_mapping).astype(np.int64)):
        if s >= 0:
            flat[s] = codes[i]
    return out


def kv_cache_write(key_cache, value_cache, key, value, positions):
    """operators/kv_cache/kv_cache_write/kv_cache_write.py:24-58: copies of the
    ``[B, H, S, D]`` caches with ``key[b, h, w]`` written at position ``positions[w]``
    (shared, 1-D) or ``positions[b, w]`` (per batch, 2-D); negative positions count
    from the end, as torch indexing does."""
    kc, vc = np.array(key_cache, copy=True), np.array(value_cache, copy=True)
    pos = np.asarray(positions, np.int64)
    b_, h_, s_, _ = kc.shape
    w_ = key.shape[2]
    for b in range(b_):
        for w in range(w_):
            p = int(pos[w] if pos.ndim == 1 else pos[b, w])
            p = p + s_ if p < 0 else p
            kc[b, :, p] = key[b, :, w]
            vc[b, :, p] = value[b, :, w]
    return kc, vc

