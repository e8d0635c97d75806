"""GPU parity of the tcgen05 W8A8 GEMM against the oracle.

The int32 accumulator and the bf16 epilogue ((acc * sa) * sb + bias, one float32 rounding per
step) are bit-exact.  The reference drop-in (int8_scaled_mm_azp: b [K, N], zero point,
azp_adj) is compared with the float64 oracle at the reference's own tolerances
(config.json: FP32 5e-4, FP16 1e-2, BF16 1.5e-2 / 1e-2).
"""
import numpy as np
import pytest
import torch

from conftest import golden_names, load_golden
from gpu_util import TORCH_DT, dev, host, require_gpu, seeded
from oracle import gemm

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _gpu():
    require_gpu()


def _ops():
    from kernelverse_b200 import ops
    return ops


def _i8(rng, shape, lo=-127, hi=128):
    return rng.integers(lo, hi, shape).astype(np.int8)


def _scales(rng, n):
    return (rng.random(n) * 9e-3 + 1e-3).astype(np.float32)


@pytest.mark.parametrize("name", golden_names("w8a8"))
def test_w8a8_golden(name):
    meta, g = load_golden(name)
    a, b = dev(g["a"][0]), dev(g["b"][0])
    acc = _ops().w8a8_int32_acc(a, b)
    np.testing.assert_array_equal(host(acc), g["acc"][0])
    out = _ops().w8a8_scaled_mm(a, b, dev(g["sa"][0]), dev(g["sb"][0]), dev(g["bias"][0], torch.bfloat16))
    np.testing.assert_array_equal(host(out), g["out"][0])


@pytest.mark.parametrize("name", golden_names("int8_scaled_mm_azp"))
def test_int8_scaled_mm_azp_golden(name):
    meta, g = load_golden(name)
    ins = [dev(g[k][0]) for k in ("a", "b", "a_scales", "b_scales", "azp_adj", "azp", "bias")]
    dt = TORCH_DT[meta["output_dtype"]]
    out = _ops().int8_scaled_mm_azp(*ins, meta["has_azp"], meta["has_bias"], dt)
    assert out.dtype == dt
    tol = {"FP32": (5e-4, 5e-4), "FP16": (1e-2, 1e-2), "BF16": (1.5e-2, 1e-2)}[meta["output_dtype"]]
    np.testing.assert_allclose(host(out), g["out"][0].astype(np.float32), rtol=tol[0], atol=tol[1])


@pytest.mark.parametrize("M,N,K", [(1, 64, 16), (16, 256, 128), (129, 300, 48), (200, 128, 8208), (256, 1000, 256),
                                   (300, 512, 1024), (5, 17, 32), (1024, 2048, 4096),
                                   # 128 < M <= 256 on CTA pairs with 256 x 448 tiles, N not a multiple of 448
                                   (256, 28672, 256), (129, 20480, 512), (200, 24576, 128), (256, 28416, 64)])
def test_w8a8_shapes_exact(M, N, K):
    rng = seeded(M * 7 + N + K)
    a, b = _i8(rng, (M, K)), _i8(rng, (N, K))
    sa, sb = _scales(rng, M), _scales(rng, N)
    bias = (0.1 * rng.standard_normal(N)).astype(np.float32)
    from oracle.numerics import round_bf16
    bias = round_bf16(bias)
    at, bt = dev(a), dev(b)
    acc = _ops().w8a8_int32_acc(at, bt)
    ref_acc = gemm.w8a8_acc(a, b)
    np.testing.assert_array_equal(host(acc), ref_acc)
    out = _ops().w8a8_scaled_mm(at, bt, dev(sa), dev(sb), dev(bias, torch.bfloat16))
    np.testing.assert_array_equal(host(out), gemm.w8a8_scaled_mm(a, b, sa, sb, bias, "BF16", acc=ref_acc))


@pytest.mark.parametrize("M", [16, 256, 4096])
def test_w8a8_baseline_config_full_size(M):
    """BASELINE third config: K = 8192, N = 28672; bit-exact oracle rows + full int32 check."""
    N, K = 28672, 8192
    rng = seeded(M)
    a, b = _i8(rng, (M, K)), _i8(rng, (N, K))
    sa, sb = _scales(rng, M), _scales(rng, N)
    from oracle.numerics import round_bf16
    bias = round_bf16((0.1 * rng.standard_normal(N)).astype(np.float32))
    at, bt = dev(a), dev(b)
    out = _ops().w8a8_scaled_mm(at, bt, dev(sa), dev(sb), dev(bias, torch.bfloat16))
    rows = np.unique(np.concatenate([np.arange(min(M, 8)), rng.integers(0, M, 24)]))
    ref = gemm.w8a8_scaled_mm(a[rows], b, sa[rows], sb, bias, "BF16")
    np.testing.assert_array_equal(host(out)[rows], ref)
    # every accumulator, checked against the library int8 GEMM (cuBLASLt via torch._int_mm)
    acc = _ops().w8a8_int32_acc(at, bt)
    if M > 16:
        assert torch.equal(acc, torch._int_mm(at, bt.t()))
    else:
        pad = torch.zeros((32, K), dtype=torch.int8, device="cuda")
        pad[:M] = at
        assert torch.equal(acc, torch._int_mm(pad, bt.t())[:M])


@pytest.mark.parametrize("dt", ["FP32", "FP16", "BF16"])
@pytest.mark.parametrize("has_azp,has_bias", [(True, True), (False, True), (True, False), (False, False)])
def test_int8_scaled_mm_azp_kn_layout(dt, has_azp, has_bias):
    rng = seeded(3)
    M, N, K = 300, 1000, 2048
    a = rng.integers(-64, 64, (M, K)).astype(np.int8)
    b = rng.integers(-64, 64, (K, N)).astype(np.int8)
    sa = (rng.random(M) * 0.02 + 0.001).astype(np.float32)
    sb = (rng.random(N) * 0.02 + 0.001).astype(np.float32)
    adj = (rng.standard_normal(N) * 0.01).astype(np.float32)
    azp = rng.integers(-8, 8, N).astype(np.float32)
    bias = (rng.standard_normal(N) * 0.01).astype(np.float32)
    out = _ops().int8_scaled_mm_azp(dev(a), dev(b), dev(sa), dev(sb), dev(adj), dev(azp), dev(bias), has_azp, has_bias,
                                    TORCH_DT[dt])
    ref = gemm.int8_scaled_mm_azp(a, b, sa, sb, adj, azp, bias, has_azp, has_bias, dt)
    tol = {"FP32": (5e-4, 5e-4), "FP16": (1e-2, 1e-2), "BF16": (1.5e-2, 1e-2)}[dt]
    np.testing.assert_allclose(host(out), ref, rtol=tol[0], atol=tol[1])


def test_w8a8_rejects_bad_k():
    from kernelverse_b200 import _lib
    a = torch.zeros((4, 24), dtype=torch.int8, device="cuda")
    with pytest.raises(_lib.KvbError, match="multiple of 16"):
        _ops().w8a8_int32_acc(a, a)


def _act_check(out, ref):
    """Gated epilogue: float32 silu on the rounded GEMM values; CUDA's and numpy's exp may differ
    in the last bit, which can move a bf16 rounding by one step."""
    o, r = host(out).astype(np.float64), np.asarray(ref, np.float64)
    np.testing.assert_allclose(o, r, rtol=8e-3, atol=1e-6)
    assert np.mean(o == r) > 0.99


@pytest.mark.parametrize("name", golden_names("w8a8_act"))
def test_w8a8_act_golden(name):
    meta, g = load_golden(name)
    bf = torch.bfloat16
    b, sb, bias = _ops().gated_weight_layout(dev(g["b_first"][0]), dev(g["b_second"][0]), dev(g["s_first"][0]),
                                             dev(g["s_second"][0]), dev(g["bias_first"][0], bf),
                                             dev(g["bias_second"][0], bf))
    out = _ops().w8a8_scaled_mm_act(dev(g["a"][0]), b, dev(g["sa"][0]), sb, bias, meta["act"])
    assert out.shape == (meta["M"], meta["I"]) and out.dtype == bf
    _act_check(out, g["out"][0])


@pytest.mark.parametrize("act", ["swiglu", "mul_and_silu"])
@pytest.mark.parametrize("M,I,K", [(1, 128, 64), (16, 384, 256), (128, 256, 1024), (129, 512, 128),
                                   (300, 1024, 512), (1024, 1280, 2048)])
def test_w8a8_act_shapes(act, M, I, K):
    """Single-CTA (M <= 128) and CTA-pair tiles, ragged M, several tile columns."""
    rng = seeded(M * 3 + I + K)
    a, b1, b2 = _i8(rng, (M, K)), _i8(rng, (I, K)), _i8(rng, (I, K))
    sa, s1, s2 = _scales(rng, M), _scales(rng, I), _scales(rng, I)
    from oracle.numerics import round_bf16
    bias1 = round_bf16((0.1 * rng.standard_normal(I)).astype(np.float32))
    bias2 = round_bf16((0.1 * rng.standard_normal(I)).astype(np.float32))
    bf = torch.bfloat16
    b, sb, bias = _ops().gated_weight_layout(dev(b1), dev(b2), dev(s1), dev(s2), dev(bias1, bf), dev(bias2, bf))
    out = _ops().w8a8_scaled_mm_act(dev(a), b, dev(sa), sb, bias, act)
    _act_check(out, gemm.w8a8_scaled_mm_act(a, b1, b2, sa, s1, s2, bias1, bias2, act, "BF16"))


def test_w8a8_act_rejects_unaligned_width():
    rng = seeded(2)
    a, b = dev(_i8(rng, (4, 64))), dev(_i8(rng, (384, 64)))     # 384 rows: not a multiple of 256
    with pytest.raises(Exception, match="multiple of 256"):
        _ops().w8a8_scaled_mm_act(a, b, dev(_scales(rng, 4)), dev(_scales(rng, 384)))
