"""Fused column-sharded TP W8A8 GEMM + all-gather on N GPUs vs the single-GPU GEMM (bit-exact),
with and without the gated (SwiGLU) epilogue.

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


def main():
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    ok = True
    try:
        for (M, N, K) in ((300, 2048, 1024), (4096, 8192, 2048)):
            g = torch.Generator(device=dev).manual_seed(M)          # same tensors on every rank
            a = torch.randint(-127, 128, (M, K), generator=g, device=dev, dtype=torch.int8)
            b = torch.randint(-127, 128, (N, K), generator=g, device=dev, dtype=torch.int8)
            sa = torch.rand((M,), generator=g, device=dev) * 9e-3 + 1e-3
            sb = torch.rand((N,), generator=g, device=dev) * 9e-3 + 1e-3
            bias = (0.1 * torch.randn((N,), generator=g, device=dev)).to(torch.bfloat16)
            n0, nw = column_shard(N, world, rank)
            tp = TPW8A8(dist.group.WORLD, M, b[n0:n0 + nw], sb[n0:n0 + nw], bias[n0:n0 + nw])
            ref = ops.w8a8_scaled_mm(a, b, sa, sb, bias)
            for _ in range(2):                                        # reuse of the symmetric buffer
                out = tp(a, sa)
                torch.cuda.synchronize()
                ok = ok and torch.equal(out, ref)
            dist.barrier()
            if rank == 0 and not ok:
                print(f"mismatch in the plain case M={M} N={N}", flush=True)
        # gated (SwiGLU) epilogue: rank r holds rows [r I/g, (r+1) I/g) of the gate and up weights
        for (M, I, K) in ((200, 256 * world, 512), (4096, 1024 * world, 1024)):
            g = torch.Generator(device=dev).manual_seed(M + 7)
            a = torch.randint(-127, 128, (M, K), generator=g, device=dev, dtype=torch.int8)
            b1 = torch.randint(-127, 128, (I, K), generator=g, device=dev, dtype=torch.int8)
            b2 = torch.randint(-127, 128, (I, K), generator=g, device=dev, dtype=torch.int8)
            sa = torch.rand((M,), generator=g, device=dev) * 9e-3 + 1e-3
            s1 = torch.rand((I,), generator=g, device=dev) * 9e-3 + 1e-3
            s2 = torch.rand((I,), generator=g, device=dev) * 9e-3 + 1e-3
            c1 = (0.1 * torch.randn((I,), generator=g, device=dev)).to(torch.bfloat16)
            c2 = (0.1 * torch.randn((I,), generator=g, device=dev)).to(torch.bfloat16)
            bl, sl_, cl = ops.gated_weight_layout(b1, b2, s1, s2, c1, c2)
            ref = ops.w8a8_scaled_mm_act(a, bl, sa, sl_, cl, act="swiglu")
            i0, iw = column_shard(I, world, rank, align=128)
            sl = slice(i0, i0 + iw)
            bs, ss, cs = ops.gated_weight_layout(b1[sl], b2[sl], s1[sl], s2[sl], c1[sl], c2[sl])
            tp = TPW8A8(dist.group.WORLD, M, bs, ss, cs, act="swiglu")
            for _ in range(2):
                out = tp(a, sa)
                torch.cuda.synchronize()
                ok = ok and torch.equal(out, ref)
            dist.barrier()
            if rank == 0 and not ok:
                print(f"mismatch in the gated case M={M} I={I}", flush=True)
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
