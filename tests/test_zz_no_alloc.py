"""kvb_paged_attention_noalloc: the allocation-free decode entry point, called through the C ABI.

For callers that cannot allocate device memory (a plugin given only its input and
output buffers, or a serving loop that must not call cudaMalloc on its hot path) the
library keeps the split-KV scratch in a static device array.  This test calls that
entry point twice in a row and checks each result against kvb_paged_attention, which
takes a caller-allocated workspace, with the decode tests' tolerance
(|err| <= 1e-2 + 1e-2 |ref|); it also checks that a call needing more than the static
scratch is rejected with KVB_E_WORKSPACE.  This file is collected last so that a run
stopping at the first failure has run every other test already; it also passes alone
in a fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

from gpu_util import require_gpu

pytestmark = pytest.mark.gpu


def _e4m3(rng, shape, scale):
    return (torch.from_numpy(rng.standard_normal(shape).astype(np.float32)) / scale).clamp(-448, 448).to(
        torch.float8_e4m3fn)


def _case(seed=7, B=16, hq=32, hkv=8, D=128, bs=16):
    rng = np.random.default_rng(seed)
    lens = rng.integers(1, 3000, B).astype(np.int32)
    maxb = int((lens.max() + bs - 1) // bs)
    nblocks = B * maxb + 4
    bt = rng.permutation(nblocks)[: B * maxb].astype(np.int32).reshape(B, maxb)
    k_scale = torch.from_numpy((rng.random(hkv) * 0.01 + 0.005).astype(np.float32))
    v_scale = torch.from_numpy((rng.random(hkv) * 0.01 + 0.005).astype(np.float32))
    kc = _e4m3(rng, (nblocks, bs, hkv, D), k_scale[None, None, :, None])
    vc = _e4m3(rng, (nblocks, bs, hkv, D), v_scale[None, None, :, None])
    q = torch.from_numpy(rng.standard_normal((B, hq, D)).astype(np.float32)).to(torch.bfloat16)
    cuda = lambda t: t.contiguous().cuda()  # noqa: E731
    return dict(q=cuda(q), kc=cuda(kc), vc=cuda(vc), ks=cuda(k_scale), vs=cuda(v_scale),
                lens=cuda(torch.from_numpy(lens)), bt=cuda(torch.from_numpy(bt)), B=B, hq=hq, hkv=hkv, D=D, bs=bs,
                nblocks=nblocks, max_len=maxb * bs)


def _common_args(c, out, part):
    from kernelverse_b200 import _lib
    return [c["q"].data_ptr(), _lib.BF16, c["kc"].data_ptr(), c["vc"].data_ptr(), _lib.E4M3, c["ks"].data_ptr(),
            c["vs"].data_ptr(), c["lens"].data_ptr(), _lib.I32, c["bt"].data_ptr(), c["bt"].shape[1], c["B"], c["hq"],
            c["hkv"], c["D"], c["bs"], c["nblocks"], c["max_len"], c["D"] ** -0.5, None, None, 0, part,
            out.data_ptr(), _lib.BF16, None, None, None, 0]


def test_noalloc_matches_workspace_entry_point_twice():
    require_gpu()
    from kernelverse_b200 import _lib
    torch.cuda.set_device(0)
    c = _case()
    part = 512
    stream = torch.cuda.current_stream().cuda_stream
    pmax = -(-c["max_len"] // part)
    ws_bytes = _lib.lib().kvb_paged_attention_workspace_size(c["B"], c["hq"], c["D"], pmax)
    assert ws_bytes <= 16 * 1024 * 1024
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
    ref = torch.empty((c["B"], c["hq"], c["D"]), dtype=torch.bfloat16, device="cuda")
    _lib.call("kvb_paged_attention", *_common_args(c, ref, part), ws.data_ptr(), ws_bytes, stream)
    for _ in range(2):
        out = torch.full_like(ref, float("nan"))
        _lib.call("kvb_paged_attention_noalloc", *_common_args(c, out, part), stream)
        torch.cuda.synchronize()
        got, want = out.float().cpu().numpy(), ref.float().cpu().numpy()
        assert np.isfinite(got).all()
        np.testing.assert_allclose(got, want, rtol=1e-2, atol=1e-2)
    assert _lib.lib().kvb_device_status(1) == 0


def test_noalloc_rejects_calls_beyond_its_scratch():
    require_gpu()
    from kernelverse_b200 import _lib
    c = _case(B=4)
    out = torch.empty((c["B"], c["hq"], c["D"]), dtype=torch.bfloat16, device="cuda")
    args = _common_args(c, out, 16)
    args[17] = 1 << 22          # max_seq_len of 4M tokens in 16-token partitions: far beyond 16 MiB of partials
    with pytest.raises(_lib.KvbError) as e:
        _lib.call("kvb_paged_attention_noalloc", *args, torch.cuda.current_stream().cuda_stream)
    assert e.value.code == 7 and "static scratch" in str(e.value)
