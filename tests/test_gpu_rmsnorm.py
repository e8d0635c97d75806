"""GPU parity of residual-add + RMSNorm (+ fused per-row quantisation) against the oracle.

Tolerances: the kernel sums s^2 in float32 in its own order, so rsqrt may differ from
the oracle by an ulp.  Hence: the updated residual is bit-exact; y / the drop-in output
within 2e-6 relative for float32 (one rounding step in the output dtype otherwise);
scales within 1e-6 relative; e4m3 codes within one e4m3 ulp (>= 99.9% exact); int8
codes within 1 (>= 99.9% exact).
"""
import numpy as np
import pytest
import torch

from conftest import golden_names, load_golden
from gpu_util import TORCH_DT, bf16_normal, dev, host, require_gpu, seeded
from oracle import numerics, rmsnorm

pytestmark = pytest.mark.gpu

OUT_TOL = {"FP32": 2e-6, "FP16": 1e-3, "BF16": 8e-3}


@pytest.fixture(autouse=True)
def _gpu():
    require_gpu()


def _ops():
    from kernelverse_b200 import ops
    return ops


@pytest.mark.parametrize("name", [n for n in golden_names("add_rmsnorm") if "fp8" not in n])
def test_add_rmsnorm_golden(name):
    meta, g = load_golden(name)
    dt = TORCH_DT[meta["dtype"]]
    out = _ops().add_rmsnorm(dev(g["x"][0], dt), dev(g["residual"][0], dt), dev(g["weight"][0], dt), meta["eps"])
    assert out.dtype == dt and tuple(out.shape) == g["out"][0].shape
    tol = OUT_TOL[meta["dtype"]]
    np.testing.assert_allclose(host(out), g["out"][0].astype(np.float32), rtol=tol, atol=tol)


@pytest.mark.parametrize("name", golden_names("add_rmsnorm_fp8"))
def test_add_rmsnorm_fp8_golden(name):
    meta, g = load_golden(name)
    bf = torch.bfloat16
    r_out, codes, scales = _ops().add_rmsnorm_quant(dev(g["x"][0], bf), dev(g["residual"][0], bf),
                                                    dev(g["weight"][0], bf), meta["eps"])
    np.testing.assert_array_equal(host(r_out), g["residual_out"][0])
    np.testing.assert_allclose(host(scales), g["scales"][0], rtol=1e-6)
    d = np.abs(numerics.e4m3_ordinal(host(codes)) - numerics.e4m3_ordinal(g["codes"][0]))
    assert d.max() <= 1 and np.mean(d == 0) >= 0.999


def _c2_inputs(rng, m, h):
    return bf16_normal(rng, (m, h)), bf16_normal(rng, (m, h)), bf16_normal(rng, (h,), std=0.02, mean=1.0)


def _check_fused(x, r, w, got, code_kind="e4m3"):
    r_out, codes, scales = got
    rr, rc, rs, _ = rmsnorm.add_rmsnorm_quant(x, r, w, 1e-6, code_kind)
    np.testing.assert_array_equal(host(r_out), rr)
    np.testing.assert_allclose(host(scales), rs, rtol=1e-6)
    c = host(codes)
    if code_kind == "e4m3":
        d = np.abs(numerics.e4m3_ordinal(c) - numerics.e4m3_ordinal(rc))
    else:
        d = np.abs(c.astype(np.int32) - rc.astype(np.int32))
    assert d.max() <= 1 and np.mean(d == 0) >= 0.999


@pytest.mark.parametrize("m,h", [(64, 8192), (5, 4096), (3, 1000), (2, 64), (1, 40000), (300, 128)])
def test_fused_fp8_shapes(m, h):
    x, r, w = _c2_inputs(seeded(m + h), m, h)
    bf = torch.bfloat16
    _check_fused(x, r, w, _ops().add_rmsnorm_quant(dev(x, bf), dev(r, bf), dev(w, bf), 1e-6))


def test_fused_int8_codes():
    x, r, w = _c2_inputs(seeded(5), 32, 4096)
    bf = torch.bfloat16
    got = _ops().add_rmsnorm_quant(dev(x, bf), dev(r, bf), dev(w, bf), 1e-6, quant_dtype=torch.int8)
    _check_fused(x, r, w, got, "int8")


def test_fused_inplace_residual():
    x, r, w = _c2_inputs(seeded(6), 16, 8192)
    bf = torch.bfloat16
    rt = dev(r, bf)
    r_out, codes, scales = _ops().add_rmsnorm_quant(dev(x, bf), rt, dev(w, bf), 1e-6, inplace_residual=True)
    assert r_out.data_ptr() == rt.data_ptr()
    _check_fused(x, r, w, (r_out, codes, scales))


def test_fused_baseline_config_full_size():
    """BASELINE second config [8192, 8192]: exact oracle on a 512-row slice, properties on all rows."""
    m = h = 8192
    rng = seeded(2)
    x, r, w = _c2_inputs(rng, m, h)
    bf = torch.bfloat16
    xt, rt, wt = dev(x, bf), dev(r, bf), dev(w, bf)
    r_out, codes, scales = _ops().add_rmsnorm_quant(xt, rt, wt, 1e-6)
    sl = slice(4096, 4608)
    _check_fused(x[sl], r[sl], w, (r_out[sl], codes[sl], scales[sl]))
    # whole-tensor properties: residual_out == bf16(x + r); |dequant - y| within half an e4m3 ulp of y
    assert torch.equal(r_out, (xt.float() + rt.float()).to(bf))
    s = xt.float() + rt.float()
    y = s * torch.rsqrt(s.pow(2).mean(-1, keepdim=True) + 1e-6) * wt.float()
    deq = codes.float() * scales[:, None]
    err = (deq - y).abs()
    bound = torch.maximum(y.abs() * 2.0 ** -4, scales[:, None] * 2.0 ** -10) * 1.01
    assert bool((err <= bound).all())
    assert bool((codes.float().abs().amax(-1) == 448.0).all())   # the row max maps to the e4m3 max


@pytest.mark.parametrize("dt", ["FP32", "FP16", "BF16"])
@pytest.mark.parametrize("shape", [[128, 4096], [16, 1, 4096], [2, 16, 64, 32], [3, 777], [1, 8192]])
def test_add_rmsnorm_shapes(dt, shape):
    rng = seeded(len(shape) + shape[-1])
    tdt = TORCH_DT[dt]
    x = dev((rng.random(shape) * 2 - 1).astype(np.float32), tdt)
    r = dev((rng.random(shape) * 2 - 1).astype(np.float32), tdt)
    w = dev(np.ones(shape[-1], np.float32), tdt)
    out = _ops().add_rmsnorm(x, r, w, 1e-6)
    ref = rmsnorm.add_rmsnorm(host(x), host(r), host(w), 1e-6, dt)
    tol = OUT_TOL[dt]
    np.testing.assert_allclose(host(out), ref, rtol=tol, atol=tol)


@pytest.mark.parametrize("kind", ["e4m3", "int8"])
def test_fused_tiny_values_quantise_to_zero(kind):
    """Rows whose normalised values span from ordinary magnitudes down to far below the
    FMA-division threshold: the tiny ones must give (signed) zero codes, as the oracle does."""
    rng = seeded(21)
    m, h = 8, 4096
    x = bf16_normal(rng, (m, h))
    tiny = numerics.round_bf16(np.array([1e-30, -1e-30, 1e-36, -1e-36, 0.0, -0.0], np.float32))
    mask = rng.random((m, h)) < 0.5
    x = np.where(mask, rng.choice(tiny, (m, h)), x).astype(np.float32)
    r = np.zeros((m, h), np.float32)
    w = bf16_normal(rng, (h,), std=0.02, mean=1.0)
    bf = torch.bfloat16
    qd = torch.float8_e4m3fn if kind == "e4m3" else torch.int8
    got = _ops().add_rmsnorm_quant(dev(x, bf), dev(r, bf), dev(w, bf), 1e-6, quant_dtype=qd)
    _check_fused(x, r, w, got, kind)
    codes = host(got[1])
    small = np.abs(x) < 1e-20
    if kind == "e4m3":
        assert np.all((codes.view(np.uint8)[small] & 0x7F) == 0)
    else:
        assert np.all(codes[small] == 0)


@pytest.mark.parametrize("m,h,chunk,qd", [(3000, 4096, 512, torch.float8_e4m3fn), (7, 8192, 1024, torch.float8_e4m3fn),
                                         (1024, 2048, 1024, torch.float8_e4m3fn), (1500, 4096, 1024, torch.int8)])
def test_fused_host_pipeline_matches_device_op(m, h, chunk, qd):
    """Host buffers in and out through row chunks on several streams (ragged last chunk, a single
    short chunk, exact chunks, int8 codes): the results equal the device op's bit for bit."""
    x, r, w = _c2_inputs(seeded(m + h + chunk), m, h)
    bf = torch.bfloat16
    hx = torch.from_numpy(x).to(bf).pin_memory()
    hr = torch.from_numpy(r).to(bf).pin_memory()
    hw = torch.from_numpy(w).to(bf)
    ro, codes, scales = _ops().add_rmsnorm_quant_host(hx, hr, hw, 1e-6, quant_dtype=qd, chunk_rows=chunk)
    torch.cuda.synchronize()
    assert not ro.is_cuda and not codes.is_cuda and not scales.is_cuda and codes.dtype == qd
    d_ro, d_codes, d_scales = _ops().add_rmsnorm_quant(hx.cuda(), hr.cuda(), hw.cuda(), 1e-6, quant_dtype=qd)
    assert torch.equal(ro, d_ro.cpu())
    assert torch.equal(codes.view(torch.uint8), d_codes.cpu().view(torch.uint8))
    assert torch.equal(scales, d_scales.cpu())
