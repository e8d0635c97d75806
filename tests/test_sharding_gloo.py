"""Multi-rank host logic on CPU (gloo, world size 2): the sharded hot path reassembles into
exactly the single-rank result.  Per-rank compute uses the numpy oracle."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from kernelverse_b200.sharding import balance_sequences, column_shard, row_shard

WORLD = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=WORLD, timeout=timedelta(seconds=60))
    try:
        from oracle import attention, gemm, numerics, rmsnorm
        rng = np.random.default_rng(0)           # identical inputs on every rank
        # 1) column-sharded W8A8: each rank fills its columns of an [M, N] buffer (as the fused
        #    epilogue does in every rank's buffer); the sum over ranks is the full product.
        M, N, K = 24, 64, 96
        a = rng.integers(-127, 128, (M, K)).astype(np.int8)
        b = rng.integers(-127, 128, (N, K)).astype(np.int8)
        sa = (rng.random(M) * 9e-3 + 1e-3).astype(np.float32)
        sb = (rng.random(N) * 9e-3 + 1e-3).astype(np.float32)
        bias = numerics.round_bf16((0.1 * rng.standard_normal(N)).astype(np.float32))
        n0, nw = column_shard(N, WORLD, rank)
        part = np.zeros((M, N), np.float32)
        part[:, n0:n0 + nw] = gemm.w8a8_scaled_mm(a, b[n0:n0 + nw], sa, sb[n0:n0 + nw], bias[n0:n0 + nw], "BF16")
        t = torch.from_numpy(part)
        dist.all_reduce(t)
        ok_gemm = np.array_equal(t.numpy(), gemm.w8a8_scaled_mm(a, b, sa, sb, bias, "BF16"))

        # 2) row-sharded add + RMSNorm + FP8: gather the rows back
        x = numerics.round_bf16(rng.standard_normal((10, 256)).astype(np.float32))
        r = numerics.round_bf16(rng.standard_normal((10, 256)).astype(np.float32))
        w = numerics.round_bf16((1 + 0.02 * rng.standard_normal(256)).astype(np.float32))
        lo, hi = row_shard(10, WORLD, rank)
        _, codes, scales, _ = rmsnorm.add_rmsnorm_quant(x[lo:hi], r[lo:hi], w, 1e-6)
        buf = np.zeros((10, 256), np.float32)
        buf[lo:hi] = codes.astype(np.float32)
        tb = torch.from_numpy(buf)
        dist.all_reduce(tb)
        _, full_codes, _, _ = rmsnorm.add_rmsnorm_quant(x, r, w, 1e-6)
        ok_rows = np.array_equal(tb.numpy(), full_codes.astype(np.float32))

        # 3) decode sequences balanced by context length
        lens = [37, 5, 90, 64, 12, 33, 70]
        bs, hq, hkv, d = 16, 4, 2, 16
        maxb = max((L + bs - 1) // bs for L in lens)
        nblocks = len(lens) * maxb
        kc = numerics.e4m3_encode(np.clip(rng.standard_normal((nblocks, bs, hkv, d)) * 50, -448, 448).astype(np.float32))
        vc = numerics.e4m3_encode(np.clip(rng.standard_normal((nblocks, bs, hkv, d)) * 50, -448, 448).astype(np.float32))
        bt = np.arange(nblocks, dtype=np.int32).reshape(len(lens), maxb)
        q = rng.standard_normal((len(lens), hq, d)).astype(np.float32)
        ks = np.full(hkv, 0.02, np.float32)
        mine = balance_sequences(lens, WORLD)[rank]
        outbuf = np.zeros((len(lens), hq, d), np.float32)
        if len(mine):
            outbuf[mine] = attention.paged_fp8_decode(q[mine], kc, vc, ks, ks, np.array(lens)[mine], bt[mine], d ** -0.5)
        to = torch.from_numpy(outbuf)
        dist.all_reduce(to)
        ref = attention.paged_fp8_decode(q, kc, vc, ks, ks, np.array(lens), bt, d ** -0.5)
        ok_decode = np.array_equal(to.numpy(), ref)
        results.put((rank, ok_gemm, ok_rows, ok_decode))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(240)
def test_sharded_path_reassembles_exactly():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=200)
    results = [q.get(timeout=5) for _ in range(WORLD)]
    assert all(p.exitcode == 0 for p in procs)
    for rank, ok_gemm, ok_rows, ok_decode in results:
        assert ok_gemm and ok_rows and ok_decode, (rank, ok_gemm, ok_rows, ok_decode)


def test_balance_sequences_properties():
    rng = np.random.default_rng(1)
    lens = rng.integers(512, 8193, 512)
    for world in (1, 2, 4, 8):
        parts = balance_sequences(lens, world)
        allidx = np.sort(np.concatenate(parts))
        assert np.array_equal(allidx, np.arange(len(lens)))
        loads = [int(lens[p].sum()) for p in parts]
        assert max(loads) - lens.sum() / world <= lens.max()
        assert max(loads) / (lens.sum() / world) < 1.01      # BASELINE fifth config: within 1 %


def test_column_and_row_shards():
    assert column_shard(57344, 8, 3) == (3 * 7168, 7168)
    with pytest.raises(ValueError):
        column_shard(100, 8, 0)
    spans = [row_shard(10, 4, r) for r in range(4)]
    assert spans == [(0, 3), (3, 6), (6, 8), (8, 10)]


# ---------------------------------------------------------------------------------------------
# The reuse protocol of TPW8A8 emulated on CPU: processes stand for GPUs, shared-memory tensors
# for the symmetric output buffers, program order for stream order and a gloo all-reduce for the
# one-element NCCL all-reduce that ends every call.  Call k of every rank writes its column
# slice of value k into ALL ranks' buffer k % depth, then joins the all-reduce; the last rank
# reads its result only after a delay, while the others go straight on to their next call.

def _reuse_worker(rank, world, port, bufs, depth, calls, results):
    import time
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        cols = bufs.shape[-1] // world
        flag = torch.zeros(1)
        seen = []
        for k in range(calls):
            idx = k % depth
            for dest in range(world):                         # the fused epilogue's peer stores
                bufs[dest, idx, :, rank * cols:(rank + 1) * cols] = float(k)
            dist.all_reduce(flag)                             # ends the call
            if rank == world - 1:
                time.sleep(0.05)                              # a slow consumer
            seen.append(bool(torch.all(bufs[rank, idx] == float(k))))
        results.put((rank, seen))
    finally:
        dist.destroy_process_group()


def _run_reuse(depth, world=2, calls=6):
    ctx = mp.get_context("spawn")
    bufs = torch.zeros((world, depth, 4, 8 * world)).share_memory_()
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_reuse_worker, args=(r, world, port, bufs, depth, calls, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=100)
    assert all(p.exitcode == 0 for p in procs)
    return dict(q.get(timeout=5) for _ in range(world))


@pytest.mark.timeout(240)
def test_tp_output_reuse_protocol_survives_a_slow_consumer():
    from kernelverse_b200.sharding import TPW8A8
    seen = _run_reuse(TPW8A8.BUFFERS)
    assert all(all(v) for v in seen.values()), seen


@pytest.mark.timeout(240)
def test_single_output_buffer_is_overwritten_under_a_slow_consumer():
    # the planted mistake (one buffer, as before the protocol): the slow rank reads a later call
    seen = _run_reuse(1)
    assert all(seen[0])
    assert not all(seen[1]), seen
