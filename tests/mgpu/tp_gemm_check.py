"""Fused column-sharded TP W8A8 GEMM + all-gather on N GPUs vs the single-GPU GEMM (bit-exact),
with and without the gated (SwiGLU) epilogue.

Each case makes several calls in a row with DIFFERENT activations, and the last rank delays
reading every result with a device spin before it copies it out, while the other ranks go
straight on to their next call.  A call that overwrote a buffer a slower rank was still
reading would show up as a mismatch on that rank.

Run with: python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 tests/mgpu/tp_gemm_check.py
"""
import os
import sys
from datetime import timedelta
from pathlib import Path

import torch
import torch.distributed as dist

sys.path.insert(0, str(Path(__file__).resolve().parents[2]))
from kernelverse_b200 import ops  # noqa: E402
from kernelverse_b200.sharding import TPW8A8, column_shard  # noqa: E402

CALLS = 5
SPIN_CYCLES = 40_000_000      # ~20 ms at the B200's clock: far longer than one call


def run_calls(tp, acts, sa, rank, world):
    """CALLS calls with different inputs; the last rank spins before copying each result."""
    outs = []
    for a in acts:
        out = tp(a, sa)
        if rank == world - 1:
            torch.cuda._sleep(SPIN_CYCLES)
        outs.append(out.clone())
    torch.cuda.synchronize()
    return outs


def main():
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    ok = True
    try:
        for (M, N, K) in ((300, 2048, 1024), (4096, 8192, 2048)):
            g = torch.Generator(device=dev).manual_seed(M)          # same tensors on every rank
            acts = [torch.randint(-127, 128, (M, K), generator=g, device=dev, dtype=torch.int8) for _ in range(CALLS)]
            b = torch.randint(-127, 128, (N, K), generator=g, device=dev, dtype=torch.int8)
            sa = torch.rand((M,), generator=g, device=dev) * 9e-3 + 1e-3
            sb = torch.rand((N,), generator=g, device=dev) * 9e-3 + 1e-3
            bias = (0.1 * torch.randn((N,), generator=g, device=dev)).to(torch.bfloat16)
            n0, nw = column_shard(N, world, rank)
            refs = [ops.w8a8_scaled_mm(a, b, sa, sb, bias) for a in acts]
            torch.cuda.synchronize()
            tp = TPW8A8(dist.group.WORLD, M, b[n0:n0 + nw], sb[n0:n0 + nw], bias[n0:n0 + nw])
            dist.barrier()
            outs = run_calls(tp, acts, sa, rank, world)
            good = [torch.equal(o, r) for o, r in zip(outs, refs)]
            ok = ok and all(good)
            if not all(good):
                print(f"rank {rank}: mismatch in the plain case M={M} N={N}, calls {good}", flush=True)
            dist.barrier()
        # gated (SwiGLU) epilogue: rank r holds rows [r I/g, (r+1) I/g) of the gate and up weights
        for (M, I, K) in ((200, 256 * world, 512), (4096, 1024 * world, 1024)):
            g = torch.Generator(device=dev).manual_seed(M + 7)
            acts = [torch.randint(-127, 128, (M, K), generator=g, device=dev, dtype=torch.int8) for _ in range(CALLS)]
            b1 = torch.randint(-127, 128, (I, K), generator=g, device=dev, dtype=torch.int8)
            b2 = torch.randint(-127, 128, (I, K), generator=g, device=dev, dtype=torch.int8)
            sa = torch.rand((M,), generator=g, device=dev) * 9e-3 + 1e-3
            s1 = torch.rand((I,), generator=g, device=dev) * 9e-3 + 1e-3
            s2 = torch.rand((I,), generator=g, device=dev) * 9e-3 + 1e-3
            c1 = (0.1 * torch.randn((I,), generator=g, device=dev)).to(torch.bfloat16)
            c2 = (0.1 * torch.randn((I,), generator=g, device=dev)).to(torch.bfloat16)
            bl, sl_, cl = ops.gated_weight_layout(b1, b2, s1, s2, c1, c2)
            refs = [ops.w8a8_scaled_mm_act(a, bl, sa, sl_, cl, act="swiglu") for a in acts]
            torch.cuda.synchronize()
            i0, iw = column_shard(I, world, rank, align=128)
            sl = slice(i0, i0 + iw)
            bs, ss, cs = ops.gated_weight_layout(b1[sl], b2[sl], s1[sl], s2[sl], c1[sl], c2[sl])
            tp = TPW8A8(dist.group.WORLD, M, bs, ss, cs, act="swiglu")
            dist.barrier()
            outs = run_calls(tp, acts, sa, rank, world)
            good = [torch.equal(o, r) for o, r in zip(outs, refs)]
            ok = ok and all(good)
            if not all(good):
                print(f"rank {rank}: mismatch in the gated case M={M} I={I}, calls {good}", flush=True)
            dist.barrier()
        flag = torch.tensor([1.0 if ok else 0.0], device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        from kernelverse_b200 import _lib
        status = _lib.lib().kvb_device_status(1)
        if rank == 0:
            print("TP_OK" if flag.item() == 1.0 and status == 0 else f"TP_FAIL status={status}", flush=True)
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
