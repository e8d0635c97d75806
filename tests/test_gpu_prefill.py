"""GPU parity of the packed causal prefill kernel (batched_prefill_attention) against the
reference's golden outputs and the numpy oracle.

Tolerances are the reference's config.json for this operator (rtol / atol 5e-4 for float32,
1e-2 for float16, 1.5e-2 / 1e-2 for bfloat16); float32 inputs run on 3xTF32 tensor-core
products, 16-bit inputs on f16 / bf16 products with float32 accumulation, so the float32 case
is also held to 2e-5 against the float64 oracle.
"""
import numpy as np
import pytest
import torch

from conftest import golden_names, load_golden
from gpu_util import TORCH_DT, dev, host, require_gpu, seeded
from oracle import attention

pytestmark = pytest.mark.gpu

TOL = {"FP32": (5e-4, 5e-4), "FP16": (1e-2, 1e-2), "BF16": (1.5e-2, 1e-2)}


@pytest.fixture(autouse=True)
def _gpu():
    require_gpu()


def _ops():
    from kernelverse_b200 import ops
    return ops


def _indptr(lens):
    return np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)


def _run(q_lens, kv_lens, hq, hkv, d, dt, seed, scale=None):
    rng = seeded(seed)
    tq, tkv = int(sum(q_lens)), int(sum(kv_lens))
    tdt = TORCH_DT[dt]
    qt = dev(rng.standard_normal((tq, hq, d)).astype(np.float32), tdt)
    kt = dev(rng.standard_normal((tkv, hkv, d)).astype(np.float32), tdt)
    vt = dev(rng.standard_normal((tkv, hkv, d)).astype(np.float32), tdt)
    qo, kvp = _indptr(q_lens), _indptr(kv_lens)
    out = _ops().batched_prefill_attention(qt, kt, vt, dev(qo), dev(kvp), scale)
    assert out.dtype == tdt and tuple(out.shape) == (tq, hq, d)
    ref = attention.batched_prefill_attention(host(qt), host(kt), host(vt), qo, kvp, hq, hkv,
                                              d ** -0.5 if scale is None else scale)
    return host(out), ref


def _check(got, ref, dt):
    rtol, atol = TOL[dt]
    np.testing.assert_allclose(got, ref, rtol=rtol, atol=atol)
    if dt == "FP32":
        np.testing.assert_allclose(got, ref, rtol=2e-5, atol=2e-5)
    else:
        assert np.mean(np.abs(got - ref)) <= 2e-3


@pytest.mark.parametrize("name", golden_names("batched_prefill_attention"))
def test_prefill_golden(name):
    meta, g = load_golden(name)
    dt = TORCH_DT[meta["dtype"]]
    out = _ops().batched_prefill_attention(dev(g["q"][0], dt), dev(g["k"][0], dt), dev(g["v"][0], dt),
                                           dev(g["qo_indptr"][0]), dev(g["kv_indptr"][0]))
    rtol, atol = TOL[meta["dtype"]]
    np.testing.assert_allclose(host(out), g["out"][0].astype(np.float32), rtol=rtol, atol=atol)


@pytest.mark.parametrize("dt", ["FP32", "FP16", "BF16"])
@pytest.mark.parametrize("q_lens,kv_lens,hq,hkv,d", [
    ([512, 384, 256, 128], [512, 384, 256, 128], 32, 8, 128),       # the reference's default shape
    ([128, 128, 128, 128], [1024, 768, 512, 256], 8, 2, 128),       # chunked prefill with context
    ([1024, 128, 64, 32, 16, 8], [1024, 128, 64, 32, 16, 8], 8, 8, 64),   # highly ragged batch
    ([300, 65], [300, 65], 16, 1, 96),                               # MQA, head_dim 96
    ([200, 1, 63], [250, 1, 64], 8, 4, 80),                          # head_dim 80, one-row requests
])
def test_prefill_shapes(dt, q_lens, kv_lens, hq, hkv, d):
    got, ref = _run(q_lens, kv_lens, hq, hkv, d, dt, sum(q_lens) + hq * 7 + d)
    _check(got, ref, dt)


@pytest.mark.parametrize("dt", ["FP32", "BF16"])
@pytest.mark.parametrize("d", [8, 40, 72, 104, 112])
def test_prefill_head_dims(dt, d):
    """Head dims that are not a multiple of 16 run on zero-padded shared tiles."""
    got, ref = _run([70, 9], [90, 9], 4, 2, d, dt, 31 + d)
    _check(got, ref, dt)


def test_prefill_scale_and_empty_request():
    """A custom softmax scale, and a request with no query rows between two others."""
    got, ref = _run([33, 0, 17], [40, 5, 17], 4, 2, 64, "FP32", 5, scale=0.3)
    _check(got, ref, "FP32")


def test_prefill_long_sequence():
    """One 4096-token request (64 query tiles, up to 64 key tiles each) beside short ones."""
    got, ref = _run([4096, 64], [4096, 64], 4, 1, 128, "BF16", 77)
    _check(got, ref, "BF16")


def test_prefill_bad_indptr_is_flagged():
    """An indptr range past the packed tensors skips its request and sets device status bit 2."""
    from kernelverse_b200 import _lib
    tdt = torch.bfloat16
    q = torch.randn((32, 2, 64), device="cuda").to(tdt)
    k = torch.randn((32, 1, 64), device="cuda").to(tdt)
    qo = torch.tensor([0, 16, 32], dtype=torch.int32, device="cuda")
    kvp = torch.tensor([0, 16, 48], dtype=torch.int32, device="cuda")    # request 1 runs past total_kv
    out = _ops().batched_prefill_attention(q, k, k, qo, kvp)
    status = _lib.lib().kvb_device_status(1)
    assert status & 4
    ref = attention.batched_prefill_attention(host(q)[:16], host(k)[:16], host(k)[:16], np.array([0, 16]),
                                              np.array([0, 16]), 2, 1, 64 ** -0.5)
    np.testing.assert_allclose(host(out)[:16], ref, rtol=1.5e-2, atol=1e-2)


def test_prefill_rejects_bad_arguments():
    ops = _ops()
    q = torch.randn((8, 4, 64), device="cuda")
    k = torch.randn((8, 3, 64), device="cuda")
    ind = torch.tensor([0, 8], dtype=torch.int32, device="cuda")
    with pytest.raises(RuntimeError, match="num_q_heads"):
        ops.batched_prefill_attention(q, k, k, ind, ind)
    k = torch.randn((8, 2, 64), device="cuda")
    with pytest.raises(ValueError, match="int32"):
        ops.batched_prefill_attention(q, k, k, ind.long(), ind.long())
    q2 = torch.randn((8, 4, 136), device="cuda")
    k2 = torch.randn((8, 2, 136), device="cuda")
    with pytest.raises(RuntimeError, match="head_dim"):
        ops.batched_prefill_attention(q2, k2, k2, ind, ind)
