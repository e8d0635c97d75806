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


def _run(q_lens, kv_lens, hq, hkv, d, dt, seed, scale=None, variant=0):
    rng = seeded(seed)
    tq, tkv = int(sum(q_lens)), int(sum(kv_lens))
    tdt = TORCH_DT[dt]
    qt = dev(rng.standard_normal((tq, hq, d)).astype(np.float32), tdt)
    kt = dev(rng.standard_normal((tkv, hkv, d)).astype(np.float32), tdt)
    vt = dev(rng.standard_normal((tkv, hkv, d)).astype(np.float32), tdt)
    qo, kvp = _indptr(q_lens), _indptr(kv_lens)
    out = _ops().batched_prefill_attention(qt, kt, vt, dev(qo), dev(kvp), scale, _variant=variant)
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


# (dtype, 1 = mma.sync / 2 = tcgen05, one query tile per CTA / 3 = tcgen05, two query tiles per CTA)
KERNELS = [("FP32", 1), ("FP16", 1), ("BF16", 1), ("FP16", 2), ("BF16", 2), ("FP16", 3), ("BF16", 3)]


@pytest.mark.parametrize("dt,variant", KERNELS)
@pytest.mark.parametrize("q_lens,kv_lens,hq,hkv,d", [
    ([512, 384, 256, 128], [512, 384, 256, 128], 32, 8, 128),       # the reference's default shape
    ([128, 128, 128, 128], [1024, 768, 512, 256], 8, 2, 128),       # chunked prefill with context
    ([1024, 128, 64, 32, 16, 8], [1024, 128, 64, 32, 16, 8], 8, 8, 64),   # highly ragged batch
    ([300, 65], [300, 65], 16, 1, 96),                               # MQA, head_dim 96
    ([200, 1, 63], [250, 1, 64], 8, 4, 80),                          # head_dim 80, one-row requests
])
def test_prefill_shapes(dt, variant, q_lens, kv_lens, hq, hkv, d):
    got, ref = _run(q_lens, kv_lens, hq, hkv, d, dt, sum(q_lens) + hq * 7 + d, variant=variant)
    _check(got, ref, dt)


@pytest.mark.parametrize("variant", [1, 2, 3])
@pytest.mark.parametrize("q_lens,kv_lens", [([130, 1, 255], [130, 1, 400]), ([128, 128], [128, 1000]),
                                            ([7, 300], [64, 300]), ([256, 257, 129], [256, 300, 129]),
                                            ([384, 100], [1000, 100]), ([513, 640, 385], [513, 700, 385])])
def test_prefill_tile_edges(variant, q_lens, kv_lens):
    """Query and key counts one past / at / below the 128-row tiles and the 256-row blocks of the
    two-tile kernel (blocks whose second tile is empty or holds one row), one-token requests, and
    requests whose queries see far more keys than queries (chunked prefill)."""
    got, ref = _run(q_lens, kv_lens, 8, 2, 128, "BF16", 901 + sum(kv_lens), variant=variant)
    _check(got, ref, "BF16")


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


@pytest.mark.parametrize("variant", [1, 2, 3])
def test_prefill_long_sequence(variant):
    """One 4096-token request (up to 64 key tiles per query tile) beside a short one."""
    got, ref = _run([4096, 64], [4096, 64], 4, 1, 128, "BF16", 77, variant=variant)
    _check(got, ref, "BF16")


def test_prefill_variants_agree_closely():
    """Both kernels on the same inputs: the same P rounding and float32 accumulation."""
    a, ref = _run([512, 384, 256, 128], [512, 384, 256, 128], 32, 8, 128, "BF16", 3, variant=1)
    b, _ = _run([512, 384, 256, 128], [512, 384, 256, 128], 32, 8, 128, "BF16", 3, variant=2)
    c, _ = _run([512, 384, 256, 128], [512, 384, 256, 128], 32, 8, 128, "BF16", 3, variant=3)
    assert np.max(np.abs(a - b)) <= 1.6e-2
    assert np.array_equal(b, c)             # the tcgen05 kernels with one and two tiles per CTA: same arithmetic per row
    assert np.mean(np.abs(a - ref)) <= 2e-3 and np.mean(np.abs(b - ref)) <= 2e-3


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


def test_prefill_tcgen05_bad_indptr_is_flagged():
    from kernelverse_b200 import _lib
    q = torch.randn((256, 2, 64), device="cuda").to(torch.bfloat16)
    k = torch.randn((256, 1, 64), device="cuda").to(torch.bfloat16)
    qo = torch.tensor([0, 128, 256], dtype=torch.int32, device="cuda")
    kvp = torch.tensor([0, 128, 300], dtype=torch.int32, device="cuda")
    out = _ops().batched_prefill_attention(q, k, k, qo, kvp, _variant=2)
    assert _lib.lib().kvb_device_status(1) & 4
    ref = attention.batched_prefill_attention(host(q)[:128], host(k)[:128], host(k)[:128], np.array([0, 128]),
                                              np.array([0, 128]), 2, 1, 64 ** -0.5)
    np.testing.assert_allclose(host(out)[:128], ref, rtol=1.5e-2, atol=1e-2)


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
    with pytest.raises(RuntimeError, match="tcgen05"):
        ops.batched_prefill_attention(q, k, k, ind, ind, _variant=2)   # float32 has no tcgen05 kernel
