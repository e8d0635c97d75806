"""Tensor-level entry points over libkvb.so, one per hot-path operator.

Each function mirrors the forward() of the KernelVerse reference operator it
replaces (same argument order, meaning, output structure, shapes and dtypes)
and runs one or more sm_100a kernels on the current CUDA stream.  PyTorch is
used only to allocate outputs (``torch.empty``) and to hand raw pointers to the
C ABI; no arithmetic happens here and there is no CPU path: CPU tensors are
rejected.
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
