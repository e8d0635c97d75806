"""Multi-GPU partitioning of the hot path (one process per GPU, torch.distributed for plumbing).

* Rows of the quantisation / add+RMSNorm kernels and sequences of decode are independent:
  each rank processes its own share with no collective on the data path.
  ``balance_sequences`` assigns sequences to ranks greedily, longest first, by context length,
  so every rank reads about the same number of KV bytes.
* The W8A8 GEMM is column-sharded (tensor parallel): rank r holds weight rows
  [r*N/g, (r+1)*N/g) and produces those output columns.  ``TPW8A8`` fuses the all-gather into
  the GEMM: the epilogue stores every output tile into all ranks' symmetric-memory output
  buffers over NVLink (``kvb_w8a8_scaled_mm_allgather``), and a one-element NCCL all-reduce on
  the same stream orders every rank's kernel before the result is read; two output buffers
  alternate so that a call never overwrites a buffer that a slower rank may still read.
"""
from __future__ import annotations

import ctypes
from typing import List, Sequence, Tuple

import numpy as np


def row_shard(rows: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous near-equal row range [start, stop) of ``rank``."""
    base, extra = divmod(rows, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def column_shard(n_total: int, world: int, rank: int, align: int = 16) -> Tuple[int, int]:
    """(first column, width) of rank's column shard; the shards must be equal and ``align``-aligned."""
    if n_total % world or (n_total // world) % align:
        raise ValueError(f"N={n_total} must split into {world} equal shards that are multiples of {align}")
    width = n_total // world
    return rank * width, width


def balance_sequences(seq_lens: Sequence[int], world: int) -> List[np.ndarray]:
    """Greedy longest-first assignment of sequences to ranks by context length.

    Returns, per rank, the sorted indices of its sequences.  Every sequence appears exactly
    once; the heaviest rank exceeds the mean load by at most the longest sequence.
    """
    lens = np.asarray(seq_lens, np.int64)
    load = np.zeros(world, np.int64)
    owned = [[] for _ in range(world)]
    for i in np.argsort(-lens, kind="stable"):
        r = int(np.argmin(load))
        owned[r].append(int(i))
        load[r] += lens[i]
    return [np.array(sorted(o), dtype=np.int64) for o in owned]


class TPW8A8:
    """Column-sharded W8A8 GEMM whose all-gather is fused into the epilogue.

    ``b_shard`` [N/g, K] int8, ``b_scales_shard`` [N/g] float32 and ``bias_shard`` [N/g] bf16 are
    this rank's slices; ``__call__(a, a_scales)`` returns the full bf16 output [M, N], a view of
    one of two symmetric-memory buffers that successive calls alternate between.

    Reuse protocol.  Every rank's kernel stores into every rank's buffer, so a call must not
    start writing a buffer while any rank may still read it.  Call k writes buffer k % 2 and
    ends with a one-element all-reduce on the calling stream, which completes only after every
    rank's kernel of call k has finished its stores (they are fenced at system scope).  Call
    k + 1 writes the other buffer, and call k + 2 -- the next writer of buffer k % 2 -- starts on
    each rank only after that rank has passed the all-reduce of call k + 1, which in turn waits
    for every rank to have issued call k + 1.  Hence the result of call k stays intact for all
    work a rank orders on the calling stream before its next call (the usual "use the output,
    then call again" pattern); work on other streams must be ordered before that call as well.
    No extra barrier is needed: the all-reduce that publishes call k also guards the buffer
    that call k + 1 overwrites.  With ``sync=False`` the caller takes over both duties.

    With ``act`` ("swiglu" or "mul_and_silu") the shard is this rank's rows of both operand
    weights in the interleaved order of ``ops.gated_weight_layout`` (N/g a multiple of 256),
    the gated activation runs in the epilogue, and the gathered output is [M, N/2].
    """

    BUFFERS = 2          # call k writes buffer k % BUFFERS

    def __init__(self, group, M: int, b_shard, b_scales_shard, bias_shard=None, act=None):
        import torch
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm_mem

        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.b, self.sb, self.bias = b_shard.contiguous(), b_scales_shard.float().contiguous(), bias_shard
        self.n_shard, self.k = self.b.shape
        self.M = M
        self.act = act
        self.N = self.n_shard * self.world // (2 if act else 1)   # gathered output columns
        dev = self.b.device
        # two [M, N] output buffers in one symmetric allocation; M * N * 2 bytes is a multiple of
        # 16 (N is a multiple of 16), so the second buffer keeps the TMA stores' alignment
        self.bufs = symm_mem.empty((self.BUFFERS, M, self.N), dtype=torch.bfloat16, device=dev)
        self.handle = symm_mem.rendezvous(self.bufs, group)
        base = list(self.handle.buffer_ptrs)
        step = M * self.N * 2
        self._ptrs = [(ctypes.c_void_p * self.world)(*[p + i * step for p in base]) for i in range(self.BUFFERS)]
        self._flag = torch.zeros(1, dtype=torch.float32, device=dev)
        self.calls = 0

    def __call__(self, a, a_scales, sync: bool = True):
        import torch
        import torch.distributed as dist
        from . import _lib

        if a.shape != (self.M, self.k):
            raise ValueError(f"a must be [{self.M}, {self.k}]")
        a = a.contiguous()
        sa = a_scales.float().contiguous()
        stream = torch.cuda.current_stream(a.device).cuda_stream
        idx = self.calls % self.BUFFERS
        ptrs = self._ptrs[idx]
        bias_ptr = self.bias.data_ptr() if self.bias is not None else None
        bias_dt = _lib.BF16 if self.bias is not None else 0
        if self.act:
            from .ops import _ACT
            _lib.call("kvb_w8a8_scaled_mm_act_allgather", a.data_ptr(), self.b.data_ptr(), sa.data_ptr(),
                      self.sb.data_ptr(), bias_ptr, bias_dt, self.M, self.n_shard, self.k, _ACT[self.act], ptrs,
                      self.world, self.rank, self.N, _lib.BF16, stream)
        else:
            _lib.call("kvb_w8a8_scaled_mm_allgather", a.data_ptr(), self.b.data_ptr(), sa.data_ptr(),
                      self.sb.data_ptr(), bias_ptr, bias_dt, self.M, self.n_shard, self.k, ptrs, self.world,
                      self.rank, self.N, _lib.BF16, stream)
        self.calls += 1
        if sync:
            # every rank's stores of this call have landed after this, and every rank has issued
            # its consumers of the previous call's buffer (which the next call overwrites)
            dist.all_reduce(self._flag, group=self.group)
        return self.bufs[idx]
