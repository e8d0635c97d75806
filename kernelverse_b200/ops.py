"""Tensor-level entry points over libkvb.so, one per hot-path operator.

Each function mirrors the forward() of the KernelVerse reference operator it
replaces (same argument order, meaning, output structure, shapes and dtypes)
and runs one or more sm_100a kernels on the current CUDA stream.  PyTorch is
used only to allocate outputs (``torch.empty``), to copy and to hand raw
pointers to the C ABI; no arithmetic happens here and there is no CPU path: CPU
tensors are rejected, except by ``add_rmsnorm_quant_host``, which streams host
tensors through the GPU kernel.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from . import _lib
from ._lib import call

_DT = {torch.float32: _lib.F32, torch.float16: _lib.F16, torch.bfloat16: _lib.BF16, torch.int8: _lib.I8,
       torch.uint8: _lib.U8, torch.int32: _lib.I32, torch.int64: _lib.I64, torch.float8_e4m3fn: _lib.E4M3}


def kvb_dtype(t: torch.dtype) -> int:
    try:
        return _DT[t]
    except KeyError:
        raise TypeError(f"dtype {t} is not supported by libkvb") from None


def _cuda(*ts: torch.Tensor) -> torch.device:
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("kernelverse_b200 ops take CUDA tensors only (there is no CPU path)")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"tensors on different devices: {dev} vs {t.device}")
    return dev


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


_workspaces = {}


def workspace(dev: torch.device, nbytes: int) -> torch.Tensor:
    """A per-device scratch buffer, grown on demand and reused across calls (stream-ordered)."""
    key = (dev.type, dev.index)
    buf = _workspaces.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=dev)
        _workspaces[key] = buf
    return buf


# --------------------------------------------------------------------------- quantisation
def dynamic_scaled_int8_quant(x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """operators/quantization/dynamic_scaled_int8_quant/dynamic_scaled_int8_quant.py:21-26."""
    dev = _cuda(x)
    x = x.contiguous()
    qshape = (1, x.shape[0]) if x.dim() == 1 else tuple(x.shape)
    q = torch.empty(qshape, dtype=torch.int8, device=dev)
    scale = torch.empty((1,), dtype=torch.float32, device=dev)
    azp = torch.empty((1,), dtype=torch.int32, device=dev)
    ws_bytes = _lib.lib().kvb_dynamic_scaled_int8_quant_workspace_size()
    ws = workspace(dev, ws_bytes)
    call("kvb_dynamic_scaled_int8_quant", _ptr(x), kvb_dtype(x.dtype), x.numel(), _ptr(q), _ptr(scale), _ptr(azp),
         _ptr(ws), ws.numel(), _stream(dev))
    return q, scale, azp


def static_scaled_int8_quant(x: torch.Tensor, scale: torch.Tensor, azp: Optional[torch.Tensor] = None) -> torch.Tensor:
    """operators/quantization/static_scaled_int8_quant/static_scaled_int8_quant.py:28-32 (float32
    arithmetic): ``clamp(round(x / max(scale, MIN_SCALE) + azp), -127, 127)`` as int8, shape of x.
    ``scale`` is a one-element float tensor and ``azp`` a one-element integer tensor on the device."""
    dev = _cuda(x, scale, azp)
    x = x.contiguous()
    if scale.numel() != 1 or (azp is not None and azp.numel() != 1):
        raise ValueError("static_scaled_int8_quant: scale and azp must have one element")
    s = scale.reshape(1).to(torch.float32)
    z = azp.reshape(1).to(torch.int32) if azp is not None else None
    q = torch.empty(x.shape, dtype=torch.int8, device=dev)
    call("kvb_static_scaled_int8_quant", _ptr(x), kvb_dtype(x.dtype), x.numel(), _ptr(s), _ptr(z) if z is not None else None,
         _ptr(q), _stream(dev))
    return q


def per_token_group_quant_int8(x: torch.Tensor, group_size: int, eps: float) -> Tuple[torch.Tensor, torch.Tensor]:
    """operators/quantization/per_token_group_quant_int8/per_token_group_quant_int8.py:23-32."""
    dev = _cuda(x)
    if x.dim() != 2:
        raise ValueError("per_token_group_quant_int8 expects [num_tokens, hidden_dim]")
    x = x.contiguous()
    t, h = x.shape
    if group_size <= 0 or h % group_size:
        raise ValueError("hidden_dim must be divisible by group_size")
    q = torch.empty((t, h), dtype=torch.int8, device=dev)
    scales = torch.empty((t, h // group_size), dtype=torch.float32, device=dev)
    call("kvb_per_token_group_quant_int8", _ptr(x), kvb_dtype(x.dtype), t, h, group_size, float(eps), _ptr(q),
         _ptr(scales), _stream(dev))
    return q, scales


# --------------------------------------------------------------------------- residual add + RMSNorm
def add_rmsnorm(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, eps: float,
                output_dtype: Optional[torch.dtype] = None) -> torch.Tensor:
    """operators/normalization/add_rmsnorm/add_rmsnorm.py:24-35 (float32 compute)."""
    dev = _cuda(x, residual, weight)
    dt = x.dtype
    if residual.dtype != dt or weight.dtype != dt:
        residual, weight = residual.to(dt), weight.to(dt)
    if output_dtype is not None and output_dtype != dt:
        raise TypeError("add_rmsnorm computes into the input dtype")
    x, residual, weight = x.contiguous(), residual.contiguous(), weight.contiguous()
    h = x.shape[-1]
    out = torch.empty_like(x)
    call("kvb_add_rmsnorm", _ptr(x), _ptr(residual), _ptr(weight), kvb_dtype(dt), x.numel() // max(h, 1), h,
         float(eps), _ptr(out), _stream(dev))
    return out


def add_rmsnorm_quant(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, eps: float,
                      quant_dtype: torch.dtype = torch.float8_e4m3fn, inplace_residual: bool = False,
                      write_residual: bool = True):
    """Fused residual add + RMSNorm + per-row dynamic quantisation.

    Returns ``(residual_out, codes, scales)``: ``residual_out = x + residual`` in the
    input dtype (``residual`` itself when ``inplace_residual``; ``None`` when
    ``write_residual`` is false), ``codes`` in ``quant_dtype`` (float8_e4m3fn or
    int8) and ``scales`` float32 ``[rows]``.
    """
    dev = _cuda(x, residual, weight)
    x, residual, weight = x.contiguous(), residual.contiguous(), weight.contiguous()
    h = x.shape[-1]
    rows = x.numel() // max(h, 1)
    if not write_residual:
        r_out = None
    elif inplace_residual:
        r_out = residual
    else:
        r_out = torch.empty_like(x)
    codes = torch.empty(x.shape, dtype=quant_dtype, device=dev)
    scales = torch.empty(x.shape[:-1], dtype=torch.float32, device=dev)
    call("kvb_add_rmsnorm_quant", _ptr(x), _ptr(residual), _ptr(weight), kvb_dtype(x.dtype), rows, h, float(eps),
         _ptr(r_out), _ptr(codes), kvb_dtype(quant_dtype), _ptr(scales), _stream(dev))
    return r_out, codes, scales


_pipe_streams = {}
_pipe_buffers = {}


def _row_chunks(rows: int, chunk: int, edge: int):
    """Chunk sizes summing to ``rows``: ``edge, 2*edge, ...`` (below ``chunk``) at both ends when the
    rows allow it, ``chunk`` in the middle and the remainder as the last middle chunk."""
    ramp, c = [], max(1, edge)
    while c < chunk:
        ramp.append(c)
        c *= 2
    if 2 * sum(ramp) + chunk > rows:
        ramp = []
    mid = rows - 2 * sum(ramp)
    middle = [chunk] * (mid // chunk) + ([mid % chunk] if mid % chunk else [])
    return ramp + middle + ramp[::-1]


def add_rmsnorm_quant_host(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, eps: float,
                           quant_dtype: torch.dtype = torch.float8_e4m3fn, out=None, device=None,
                           chunk_rows: int = 1024, edge_rows: int = 256, slots: int = 3):
    """:func:`add_rmsnorm_quant` for host-resident ``[..., H]`` tensors, through the GPU.

    Rows travel in chunks through three CUDA streams, one per stage: copies in, kernels, copies
    out, chained chunk by chunk with events.  The copy-in stream only waits for a device buffer
    slot (``slots`` of them, reused round robin) to be copied out, so the two copy engines run
    side by side.  Chunks are ``chunk_rows`` rows, ramping up from ``edge_rows`` at the start and
    back down at the end, so the first copy in and the last copy out, which run alone, are short.
    Rows are independent, so the results equal :func:`add_rmsnorm_quant`'s.  Inputs should be
    pinned for the copies to overlap.  Returns host tensors ``(residual_out, codes, scales)``
    (into ``out`` when given); they are complete once the current stream's work is, like any
    non-blocking copy to the host.
    """
    if x.is_cuda or residual.is_cuda:
        raise ValueError("add_rmsnorm_quant_host takes host tensors; use add_rmsnorm_quant for device tensors")
    if x.shape != residual.shape or x.dtype != residual.dtype:
        raise ValueError("x and residual must have the same shape and dtype")
    if slots < 1:
        raise ValueError("add_rmsnorm_quant_host needs at least one buffer slot")
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    h = x.shape[-1]
    rows = x.numel() // max(h, 1)
    x2, r2 = x.contiguous().view(rows, h), residual.contiguous().view(rows, h)
    if out is None:
        pin = torch.cuda.is_available()
        out = (torch.empty(x.shape, dtype=x.dtype, pin_memory=pin), torch.empty(x.shape, dtype=quant_dtype, pin_memory=pin),
               torch.empty(x.shape[:-1], dtype=torch.float32, pin_memory=pin))
    h_rout, h_codes, h_scales = (t.view(rows, h) if i < 2 else t.view(rows) for i, t in enumerate(out))
    cur = torch.cuda.current_stream(dev)
    if dev.index not in _pipe_streams:
        _pipe_streams[dev.index] = tuple(torch.cuda.Stream(dev) for _ in range(3))
    s_in, s_run, s_out = _pipe_streams[dev.index]
    dw = weight.to(dev, non_blocking=True).contiguous()
    dw.record_stream(s_run)
    cr = max(1, min(chunk_rows, rows))
    # Device buffer slots kept across calls: the stage streams start after the current stream and
    # the current stream waits for them at the end, so the previous call is done with every slot
    # before this call reuses one.
    bkey = (dev.index, slots, cr, h, x.dtype, quant_dtype)
    bufs = _pipe_buffers.get(bkey)
    if bufs is None:
        bufs = [(torch.empty((cr, h), dtype=x.dtype, device=dev), torch.empty((cr, h), dtype=x.dtype, device=dev),
                 torch.empty((cr, h), dtype=x.dtype, device=dev), torch.empty((cr, h), dtype=quant_dtype, device=dev),
                 torch.empty((cr,), dtype=torch.float32, device=dev)) for _ in range(slots)]
        _pipe_buffers.clear()              # one configuration at a time
        _pipe_buffers[bkey] = bufs
    for s in (s_in, s_run, s_out):
        s.wait_stream(cur)
    copied_out = [None] * slots            # event: the slot's last chunk is back on the host
    r1 = 0
    for i, n in enumerate(_row_chunks(rows, cr, edge_rows)):
        r0, r1 = r1, r1 + n
        k = i % slots
        dx, dr, drout, dcodes, dscales = bufs[k]
        if copied_out[k] is not None:
            s_in.wait_event(copied_out[k])
        with torch.cuda.stream(s_in):
            dx[:n].copy_(x2[r0:r1], non_blocking=True)
            dr[:n].copy_(r2[r0:r1], non_blocking=True)
        s_run.wait_event(s_in.record_event())
        call("kvb_add_rmsnorm_quant", _ptr(dx), _ptr(dr), _ptr(dw), kvb_dtype(x.dtype), n, h, float(eps),
             _ptr(drout), _ptr(dcodes), kvb_dtype(quant_dtype), _ptr(dscales), s_run.cuda_stream)
        s_out.wait_event(s_run.record_event())
        with torch.cuda.stream(s_out):
            h_rout[r0:r1].copy_(drout[:n], non_blocking=True)
            h_codes[r0:r1].copy_(dcodes[:n], non_blocking=True)
            h_scales[r0:r1].copy_(dscales[:n], non_blocking=True)
        copied_out[k] = s_out.record_event()
    for s in (s_in, s_run, s_out):
        cur.wait_stream(s)
    return out


# --------------------------------------------------------------------------- paged KV cache
def _index_dtype(t: torch.Tensor) -> int:
    if t.dtype not in (torch.int32, torch.int64):
        raise TypeError("slot/sequence indices must be int32 or int64")
    return kvb_dtype(t.dtype)


def paged_kv_cache_update(to_cache: torch.Tensor, kv_cache: torch.Tensor, slot_mapping: torch.Tensor) -> torch.Tensor:
    """operators/kv_cache/paged_kv_cache_update/paged_kv_cache_update.py:21-31 (returns a new cache)."""
    dev = _cuda(to_cache, kv_cache, slot_mapping)
    kv_cache, slot_mapping = kv_cache.contiguous(), slot_mapping.contiguous()
    to_cache = to_cache.to(kv_cache.dtype).contiguous()
    out = torch.empty_like(kv_cache)
    nb, bs = kv_cache.shape[0], kv_cache.shape[1]
    slot_elems = kv_cache.numel() // max(nb * bs, 1)
    call("kvb_paged_kv_cache_update", _ptr(to_cache), _ptr(kv_cache), _ptr(out), _ptr(slot_mapping),
         _index_dtype(slot_mapping), kvb_dtype(kv_cache.dtype), slot_mapping.numel(), nb * bs, slot_elems, _stream(dev))
    return out


def kv_cache_write(key_cache: torch.Tensor, value_cache: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                   positions: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """operators/kv_cache/kv_cache_write/kv_cache_write.py:24-58 -> new (key_cache, value_cache).

    Caches [batch, heads, max_seq_len, head_dim]; key/value [batch, heads, write_len, head_dim]
    (converted to the cache dtype); positions [write_len] (shared) or [batch, write_len]."""
    dev = _cuda(key_cache, value_cache, key, value, positions)
    key_cache, value_cache = key_cache.contiguous(), value_cache.contiguous()
    if key_cache.dim() != 4 or value_cache.shape != key_cache.shape:
        raise ValueError("kv_cache_write: caches must both be [batch, heads, max_seq_len, head_dim]")
    b, h, smax, d = key_cache.shape
    key = key.to(key_cache.dtype).contiguous()
    value = value.to(key_cache.dtype).contiguous()
    if key.dim() != 4 or key.shape[:2] != (b, h) or key.shape[3] != d or value.shape != key.shape:
        raise ValueError("kv_cache_write: key/value must be [batch, heads, write_len, head_dim] like the caches")
    w = key.shape[2]
    positions = positions.contiguous()
    if positions.dim() == 1:
        per_batch = 0
        if positions.shape[0] != w:
            raise ValueError("kv_cache_write: shared positions must have write_len entries")
    elif positions.dim() == 2 and tuple(positions.shape) == (b, w):
        per_batch = 1
    else:
        raise ValueError("kv_cache_write: positions must be [write_len] or [batch, write_len]")
    k_out, v_out = torch.empty_like(key_cache), torch.empty_like(value_cache)
    call("kvb_kv_cache_write", _ptr(key), _ptr(value), _ptr(key_cache), _ptr(value_cache), _ptr(k_out), _ptr(v_out),
         _ptr(positions), _index_dtype(positions), per_batch, kvb_dtype(key_cache.dtype), b, h, smax, w, d, _stream(dev))
    return k_out, v_out


def paged_fp8_kv_write(x_new: torch.Tensor, cache: torch.Tensor, slot_mapping: torch.Tensor,
                       head_scales: torch.Tensor) -> torch.Tensor:
    """Quantise x_new [T, Hkv, D] into the e4m3 cache [num_blocks, block_size, Hkv, D] in place."""
    dev = _cuda(x_new, cache, slot_mapping, head_scales)
    x_new, slot_mapping = x_new.contiguous(), slot_mapping.contiguous()
    head_scales = head_scales.to(torch.float32).contiguous()
    t, h, d = x_new.shape
    nslots = cache.shape[0] * cache.shape[1]
    call("kvb_paged_fp8_kv_write", _ptr(x_new), kvb_dtype(x_new.dtype), _ptr(cache), _ptr(slot_mapping),
         _index_dtype(slot_mapping), _ptr(head_scales), t, nslots, h, d, _stream(dev))
    return cache


# --------------------------------------------------------------------------- decode attention
def _cache_kvb_dtype(t: torch.Tensor) -> int:
    if t.dtype in (torch.uint8, torch.float8_e4m3fn):
        return _lib.E4M3
    return kvb_dtype(t.dtype)


def _paged_attention(query, key_cache, value_cache, seq_lens, block_table, *, num_kv_heads, block_size, num_blocks,
                     max_seq_len, scale, k_scale=None, v_scale=None, k_new=None, v_new=None, partition_size=0,
                     out_dtype=None, v2=False):
    dev = _cuda(query, key_cache, value_cache, seq_lens, block_table, k_scale, v_scale, k_new, v_new)
    query = query.contiguous()
    b, hq, d = query.shape
    out_dtype = out_dtype or query.dtype
    out = torch.empty((b, hq, d), dtype=out_dtype, device=dev)
    # partition_size 0: the library's automatic size (smaller partitions for small grids)
    part = partition_size if partition_size else _lib.lib().kvb_paged_attention_auto_partition(b, int(max_seq_len))
    pmax = max(1, -(-int(max_seq_len) // part))
    es = ml = tmp = None
    if v2:
        es = torch.empty((b, hq, pmax), dtype=out_dtype, device=dev)
        ml = torch.empty((b, hq, pmax), dtype=out_dtype, device=dev)
        tmp = torch.empty((b, hq, pmax, d), dtype=out_dtype, device=dev)
    ws_bytes = _lib.lib().kvb_paged_attention_workspace_size(b, hq, d, pmax)
    ws = workspace(dev, ws_bytes)
    bt_ptr, bt_stride = None, 0
    if block_table is not None:
        block_table = block_table.to(torch.int32).contiguous()
        bt_ptr, bt_stride = block_table.data_ptr(), block_table.shape[1]
    seq_lens = seq_lens.contiguous()
    if k_scale is not None:
        k_scale = k_scale.to(torch.float32).contiguous()
        v_scale = v_scale.to(torch.float32).contiguous()
    if k_new is not None:
        k_new, v_new = k_new.contiguous(), v_new.contiguous()
    call("kvb_paged_attention", _ptr(query), kvb_dtype(query.dtype), _ptr(key_cache.contiguous()),
         _ptr(value_cache.contiguous()), _cache_kvb_dtype(key_cache), _ptr(k_scale), _ptr(v_scale), _ptr(seq_lens),
         _index_dtype(seq_lens), bt_ptr, bt_stride, b, hq, num_kv_heads, d, block_size, num_blocks, int(max_seq_len),
         float(scale), _ptr(k_new), _ptr(v_new), kvb_dtype(k_new.dtype) if k_new is not None else 0, part, _ptr(out),
         kvb_dtype(out_dtype), _ptr(es), _ptr(ml), _ptr(tmp), pmax, _ptr(ws), ws.numel(), _stream(dev))
    return (out, es, ml, tmp) if v2 else out


def paged_attention_v1(query, key_cache, value_cache, seq_lens, block_table, scale: Optional[float] = None,
                       output_dtype: Optional[torch.dtype] = None):
    """operators/attention/paged_attention_v1/paged_attention_v1.py:27-92.

    ``key_cache`` / ``value_cache`` are the reference's ``[total_blocks, Hkv, block_size, D]``
    tensors, whose memory the reference reads as ``[total_blocks, block_size, Hkv, D]``
    (reshape of a gathered block, ``:64-69``); the kernel reads the same memory the same way.
    """
    nb, hkv, bs, d = key_cache.shape
    scale = d ** -0.5 if scale is None else scale
    return _paged_attention(query, key_cache, value_cache, seq_lens, block_table, num_kv_heads=hkv, block_size=bs,
                            num_blocks=nb, max_seq_len=block_table.shape[1] * bs, scale=scale, out_dtype=output_dtype)


def paged_attention_v2(query, key_cache, value_cache, seq_lens, block_table, partition_size: int,
                       scale: Optional[float] = None, output_dtype: Optional[torch.dtype] = None):
    """operators/attention/paged_attention_v2/paged_attention_v2.py:28-175 -> (out, exp_sums, max_logits, tmp_out)."""
    nb, hkv, bs, d = key_cache.shape
    scale = d ** -0.5 if scale is None else scale
    # the partition outputs are sized by the longest sequence, as the reference's .item() does (:42-43)
    max_len = int(seq_lens.detach().to("cpu", non_blocking=False).max()) if seq_lens.numel() else 0
    return _paged_attention(query, key_cache, value_cache, seq_lens, block_table, num_kv_heads=hkv, block_size=bs,
                            num_blocks=nb, max_seq_len=max_len, scale=scale, partition_size=partition_size,
                            out_dtype=output_dtype, v2=True)


def flash_attn_with_kvcache(q, k_cache, v_cache, cache_seqlens, softmax_scale: Optional[float] = None):
    """operators/attention/flash_attn_with_kvcache/flash_attn_with_kvcache.py:29-56 ->
    (output [B, Sq, H, D] in q's dtype, softmax_lse [B, H, Sq] float32).

    q [B, Sq, H, D]; caches [B, Sk, Hkv, D] of q's dtype; cache_seqlens [B]: every query token
    of sequence b attends to its first cache_seqlens[b] keys."""
    dev = _cuda(q, k_cache, v_cache, cache_seqlens)
    b, sq, h, d = q.shape
    sk, hkv = k_cache.shape[1], k_cache.shape[2]
    if k_cache.shape != (b, sk, hkv, d) or v_cache.shape != k_cache.shape:
        raise ValueError("flash_attn_with_kvcache: caches must be [batch, seq_len_k, heads, head_dim]")
    if k_cache.dtype != q.dtype or v_cache.dtype != q.dtype:
        raise ValueError("flash_attn_with_kvcache: q and the caches must share a dtype")
    scale = d ** -0.5 if softmax_scale is None else softmax_scale
    q, k_cache, v_cache = q.contiguous(), k_cache.contiguous(), v_cache.contiguous()
    cache_seqlens = cache_seqlens.contiguous()
    out = torch.empty((b, sq, h, d), dtype=q.dtype, device=dev)
    lse = torch.empty((b, h, sq), dtype=torch.float32, device=dev)
    ws = workspace(dev, _lib.lib().kvb_flash_attn_with_kvcache_workspace_size(b, sq, h, d, sk))
    call("kvb_flash_attn_with_kvcache", _ptr(q), _ptr(k_cache), _ptr(v_cache), kvb_dtype(q.dtype), _ptr(cache_seqlens),
         _index_dtype(cache_seqlens), b, sq, sk, h, hkv, d, float(scale), _ptr(out), _ptr(lse), _ptr(ws), ws.numel(),
         _stream(dev))
    return out, lse


def batched_prefill_attention(q, k, v, qo_indptr, kv_indptr, softmax_scale: Optional[float] = None, _variant: int = 0):
    """operators/attention/batched_prefill_attention/batched_prefill_attention.py:30-73 ->
    packed output [total_q, Hq, D] in q's dtype.

    q [total_q, Hq, D]; k / v [total_kv, Hkv, D] of q's dtype; qo_indptr / kv_indptr int32
    [batch + 1] on the device: causal attention inside each request, its query rows being the
    last q_len positions of its kv_len keys; query head h reads KV head h // (Hq / Hkv)."""
    dev = _cuda(q, k, v, qo_indptr, kv_indptr)
    tq, hq, d = q.shape
    tkv, hkv = k.shape[0], k.shape[1]
    if k.shape != (tkv, hkv, d) or v.shape != k.shape:
        raise ValueError("batched_prefill_attention: k and v must be [total_kv, num_kv_heads, head_dim]")
    if k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError("batched_prefill_attention: q, k and v must share a dtype")
    if qo_indptr.dtype != torch.int32 or kv_indptr.dtype != torch.int32:
        raise ValueError("batched_prefill_attention: indptrs must be int32")
    if qo_indptr.dim() != 1 or kv_indptr.shape != qo_indptr.shape:
        raise ValueError("batched_prefill_attention: indptrs must be [batch + 1]")
    scale = d ** -0.5 if softmax_scale is None else softmax_scale
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    qo_indptr, kv_indptr = qo_indptr.contiguous(), kv_indptr.contiguous()
    out = torch.empty((tq, hq, d), dtype=q.dtype, device=dev)
    # _variant (tests): 0 = automatic kernel choice, 1 = the mma.sync kernel, 2 / 3 = the tcgen05
    # kernel with one / two query tiles per CTA
    call("kvb_batched_prefill_attention_variant", _ptr(q), _ptr(k), _ptr(v), kvb_dtype(q.dtype), _ptr(qo_indptr),
         _ptr(kv_indptr), qo_indptr.numel() - 1, tq, tkv, hq, hkv, d, float(scale), _ptr(out), int(_variant),
         _stream(dev))
    return out


_FLASH_DECODE_INDEX = {}


def _flash_decode_index(dev, b, h, sq, s, causal):
    """(block table or None, seq_lens) mapping each (batch, head, query token) of a
    [B, H, S, D] cache to one single-head sequence; cached per shape."""
    key = (dev, b, h, sq, s, causal)
    if key not in _FLASH_DECODE_INDEX:
        bt = None
        if sq > 1:   # the sq queries of (b, h) share block b * h
            bt = torch.arange(b * h, dtype=torch.int32, device=dev).repeat_interleave(sq).view(b * h * sq, 1)
        i = torch.arange(sq, dtype=torch.int32, device=dev)
        lens = (s - sq + 1 + i) if causal else torch.full((sq,), s, dtype=torch.int32, device=dev)
        _FLASH_DECODE_INDEX[key] = (bt, lens.repeat(b * h).contiguous())
    return _FLASH_DECODE_INDEX[key]


def flash_decoding_attention(query, key_cache, value_cache, chunk_size: int, causal: bool = False,
                             scale: Optional[float] = None):
    """operators/attention/flash_decoding_attention/flash_decoding_attention.py:30-87 ->
    (output [B, H, Sq, D], exp_sums [B, H, Sq, P], max_logits [B, H, Sq, P], partial_outputs
    [B, H, Sq, P, D]) with P = ceil(S / chunk_size), all in the query dtype.

    query [B, H, Sq, D]; caches [B, H, S, D] (one KV head per query head).  Every (b, h, query
    token) is one single-head sequence of the split-KV decode kernel whose partitions are the
    reference's chunks; a causal query i attends to the first S - Sq + 1 + i keys."""
    b, h, sq, d = query.shape
    s = key_cache.shape[2]
    if key_cache.shape != (b, h, s, d) or value_cache.shape != key_cache.shape:
        raise ValueError("flash_decoding_attention: caches must be [batch, heads, kv_len, head_dim]")
    dev = _cuda(query, key_cache, value_cache)
    scale = d ** -0.5 if scale is None else scale
    bt, lens = _flash_decode_index(dev, b, h, sq, s, bool(causal))
    kc = key_cache.contiguous().view(b * h, s, 1, d)
    vc = value_cache.contiguous().view(b * h, s, 1, d)
    q = query.contiguous().view(b * h * sq, 1, d)
    out, es, ml, tmp = _paged_attention(q, kc, vc, lens, bt, num_kv_heads=1, block_size=s, num_blocks=b * h,
                                        max_seq_len=s, scale=scale, partition_size=chunk_size, v2=True)
    p = es.shape[-1]
    return (out.view(b, h, sq, d), es.view(b, h, sq, p), ml.view(b, h, sq, p), tmp.view(b, h, sq, p, d))


def batched_decode_attention(q, k_cache, v_cache, seq_lens, scale: Optional[float] = None,
                             output_dtype: Optional[torch.dtype] = None):
    """operators/attention/batched_decode_attention/batched_decode_attention.py:30-52 (dense [B, L, Hkv, D])."""
    b, lmax, hkv, d = k_cache.shape
    scale = d ** -0.5 if scale is None else scale
    return _paged_attention(q, k_cache, v_cache, seq_lens, None, num_kv_heads=hkv, block_size=lmax, num_blocks=b,
                            max_seq_len=lmax, scale=scale, out_dtype=output_dtype)


def paged_fp8_decode(query, k_cache, v_cache, k_scale, v_scale, seq_lens, block_table, scale: Optional[float] = None,
                     k_new=None, v_new=None, max_seq_len: Optional[int] = None, partition_size: int = 0):
    """FP8 paged decode (BASELINE fourth config): caches [num_blocks, block_size, Hkv, D] of e4m3 codes.

    With ``k_new`` / ``v_new`` [B, Hkv, D], each sequence's token ``seq_len - 1`` is first
    quantised into its slot (``block_table[b][(L-1)//bs]*bs + (L-1)%bs``) and attended to.
    """
    nb, bs, hkv, d = k_cache.shape
    scale = d ** -0.5 if scale is None else scale
    if max_seq_len is None:
        max_seq_len = block_table.shape[1] * bs
    return _paged_attention(query, k_cache, v_cache, seq_lens, block_table, num_kv_heads=hkv, block_size=bs,
                            num_blocks=nb, max_seq_len=max_seq_len, scale=scale, k_scale=k_scale, v_scale=v_scale,
                            k_new=k_new, v_new=v_new, partition_size=partition_size, out_dtype=query.dtype)


# --------------------------------------------------------------------------- W8A8 GEMM
def _gemm(a, b, b_layout, a_scales, b_scales, bias, azp, azp_adj, out_dtype):
    dev = _cuda(a, b, a_scales, b_scales, bias, azp, azp_adj)
    a = a.contiguous()
    b = b.contiguous()
    m, k = a.shape
    n = b.shape[0] if b_layout == 0 else b.shape[1]
    out = torch.empty((m, n), dtype=out_dtype, device=dev)
    f32 = lambda t: None if t is None else t.to(torch.float32).contiguous()  # noqa: E731
    a_scales, b_scales, azp, azp_adj = f32(a_scales), f32(b_scales), f32(azp), f32(azp_adj)
    if bias is not None:
        bias = bias.contiguous()
    ws_bytes = _lib.lib().kvb_w8a8_workspace_size(m, n, k, b_layout, int(azp is not None))
    ws = workspace(dev, ws_bytes)
    call("kvb_w8a8_scaled_mm", _ptr(a), _ptr(b), b_layout, _ptr(a_scales), _ptr(b_scales), _ptr(bias),
         kvb_dtype(bias.dtype) if bias is not None else 0, _ptr(azp), _ptr(azp_adj), m, n, k, _ptr(out),
         kvb_dtype(out_dtype), n, _ptr(ws), ws.numel(), _stream(dev))
    return out


def w8a8_scaled_mm(a: torch.Tensor, b: torch.Tensor, a_scales: torch.Tensor, b_scales: torch.Tensor,
                   bias: Optional[torch.Tensor] = None, out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """BASELINE third config: out = (acc * a_scales[m]) * b_scales[n] + bias[n], acc = a[M,K] . b[N,K]^T (int32)."""
    return _gemm(a, b, 0, a_scales, b_scales, bias, None, None, out_dtype)


def w8a8_int32_acc(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """The exact int32 accumulator a[M,K] . b[N,K]^T of the W8A8 GEMM."""
    return _gemm(a, b, 0, None, None, None, None, None, torch.int32)


_ACT = {"swiglu": 1, "mul_and_silu": 2}


def gated_weight_layout(first: torch.Tensor, second: torch.Tensor, first_scales: torch.Tensor,
                        second_scales: torch.Tensor, first_bias: Optional[torch.Tensor] = None,
                        second_bias: Optional[torch.Tensor] = None):
    """One-time weight preparation for :func:`w8a8_scaled_mm_act`: the two operand weights
    [I, K] (I a multiple of 128; e.g. gate and up projections) with their per-row scales and
    biases, interleaved in blocks of 128 rows -> (b [2I, K], b_scales [2I], bias [2I] or None)."""
    i, k = first.shape
    if second.shape != (i, k) or i % 128:
        raise ValueError("gated_weight_layout: two [I, K] weights with I a multiple of 128")

    def inter(x, y):
        return torch.stack((x.reshape(i // 128, 128, *x.shape[1:]), y.reshape(i // 128, 128, *y.shape[1:])),
                           dim=1).reshape(2 * i, *x.shape[1:]).contiguous()
    bias = None
    if first_bias is not None or second_bias is not None:
        fb = first_bias if first_bias is not None else torch.zeros_like(second_bias)
        sb = second_bias if second_bias is not None else torch.zeros_like(first_bias)
        bias = inter(fb, sb)
    return inter(first, second), inter(first_scales.to(torch.float32), second_scales.to(torch.float32)), bias


def w8a8_scaled_mm_act(a: torch.Tensor, b: torch.Tensor, a_scales: torch.Tensor, b_scales: torch.Tensor,
                       bias: Optional[torch.Tensor] = None, act: str = "swiglu",
                       out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """W8A8 GEMM + gated activation in one kernel: with f = the W8A8 epilogue value rounded to
    out_dtype, out[:, c] = silu(f_first) * f_second ("swiglu", operators/activation/swiglu) or
    f_first * silu(f_second) ("mul_and_silu", operators/activation/mul_and_silu).  b, b_scales
    and bias in the interleaved order of :func:`gated_weight_layout`; out [M, N / 2]."""
    dev = _cuda(a, b, a_scales, b_scales, bias)
    a, b = a.contiguous(), b.contiguous()
    m, k = a.shape
    n = b.shape[0]
    out = torch.empty((m, n // 2), dtype=out_dtype, device=dev)
    sa = a_scales.to(torch.float32).contiguous()
    sb = b_scales.to(torch.float32).contiguous()
    if bias is not None:
        bias = bias.contiguous()
    call("kvb_w8a8_scaled_mm_act", _ptr(a), _ptr(b), _ptr(sa), _ptr(sb), _ptr(bias),
         kvb_dtype(bias.dtype) if bias is not None else 0, m, n, k, _ACT[act], _ptr(out), kvb_dtype(out_dtype), n // 2,
         _stream(dev))
    return out


def int8_scaled_mm_azp(a, b, a_scales, b_scales, azp_adj, azp, bias, has_azp: bool, has_bias: bool,
                       output_dtype: torch.dtype):
    """operators/gemm/int8_scaled_mm_azp/int8_scaled_mm_azp.py:61-85 (b is [K, N]; azp_adj always added)."""
    m, n = a.shape[0], b.shape[1]
    if a_scales.numel() != m or b_scales.numel() != n:
        raise ValueError("a_scales must have M entries and b_scales N entries")
    return _gemm(a, b, 1, a_scales.reshape(-1), b_scales.reshape(-1), bias.reshape(-1) if has_bias else None,
                 azp.reshape(-1) if has_azp else None, azp_adj.reshape(-1), output_dtype)
