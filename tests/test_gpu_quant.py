"""GPU parity of the int8 quantisation kernels against the oracle: bit-exact codes and scales."""
import numpy as np
import pytest
import torch

from conftest import golden_names, load_golden
from gpu_util import TORCH_DT, bf16_normal, dev, host, require_gpu, seeded
from oracle import quant

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _gpu():
    require_gpu()


def _ops():
    from kernelverse_b200 import ops
    return ops


@pytest.mark.parametrize("name", golden_names("dynamic_scaled_int8_quant"))
def test_dynamic_quant_golden(name):
    meta, g = load_golden(name)
    x, xdt = g["x"]
    q, s, azp = _ops().dynamic_scaled_int8_quant(dev(x, TORCH_DT[xdt]))
    np.testing.assert_array_equal(host(s), g["scale"][0])
    np.testing.assert_array_equal(host(q), g["q"][0])
    np.testing.assert_array_equal(host(azp), [0])


@pytest.mark.parametrize("name", golden_names("per_token_group_quant_int8"))
def test_group_quant_golden(name):
    meta, g = load_golden(name)
    x, xdt = g["x"]
    q, s = _ops().per_token_group_quant_int8(dev(x, TORCH_DT[xdt]), meta["group_size"], meta["eps"])
    np.testing.assert_array_equal(host(s), g["scales"][0])
    np.testing.assert_array_equal(host(q), g["q"][0])


def baseline_c1_input(rng, m=2048, k=4096):
    """BASELINE first config: bf16 N(0,1) with 0.1% of entries x50."""
    x = rng.standard_normal((m, k)).astype(np.float32)
    idx = rng.choice(x.size, size=x.size // 1000, replace=False)
    x.reshape(-1)[idx] *= 50.0
    from oracle.numerics import round_bf16
    return round_bf16(x)


def test_per_token_quant_baseline_config_full_size():
    x = baseline_c1_input(seeded(1))
    q, s = _ops().per_token_group_quant_int8(dev(x, torch.bfloat16), 4096, 1e-6)
    rq, rs = quant.per_token_group_quant_int8(x, 4096, 1e-6)
    np.testing.assert_array_equal(host(s)[:, 0], rs[:, 0])
    np.testing.assert_array_equal(host(q), rq)


@pytest.mark.parametrize("dt", ["FP32", "FP16", "BF16"])
@pytest.mark.parametrize("t,h,g", [(64, 4096, 128), (33, 256, 32), (5, 11008, 64), (7, 96, 96), (3, 100, 100),
                                   (4, 8192, 8192), (2, 40, 8), (3, 96, 48), (1, 70000, 70000),
                                   # many per-token rows: 1, 2 and 4 vectors per thread of the row-block kernel
                                   (320, 1024, 1024), (297, 4096, 4096), (600, 8192, 8192), (1000, 2048, 2048),
                                   # team kernel: 1, 2, 4, 8 and 16 warps a group, partial last CTA
                                   (149, 4096, 4096), (5000, 4096, 4096), (3000, 8192, 8192), (40, 512, 512),
                                   (50, 16384, 16384), (7, 4096, 2048), (33, 1536, 768)])
def test_group_quant_shapes(dt, t, h, g):
    rng = seeded(t * 7 + h)
    x = (rng.standard_normal((t, h)) * 3).astype(np.float32)
    xt = dev(x, TORCH_DT[dt])
    x = host(xt).astype(np.float32)
    x[0, : min(h, g)] = 0.0                         # an all-zero group -> scale = eps
    xt = dev(x, TORCH_DT[dt])
    q, s = _ops().per_token_group_quant_int8(xt, g, 1e-6)
    rq, rs = quant.per_token_group_quant_int8(x, g, 1e-6)
    np.testing.assert_array_equal(host(s), rs)
    np.testing.assert_array_equal(host(q), rq)


def test_group_quant_misaligned_input_uses_scalar_path():
    rng = seeded(3)
    base = dev(rng.standard_normal(16 * 64 + 1).astype(np.float32), torch.bfloat16)
    x = base[1:].view(16, 64)                        # 2-byte offset: not 16-byte aligned
    assert x.data_ptr() % 16 != 0
    q, s = _ops().per_token_group_quant_int8(x, 64, 1e-6)
    rq, rs = quant.per_token_group_quant_int8(host(x).astype(np.float32), 64, 1e-6)
    np.testing.assert_array_equal(host(q), rq)
    np.testing.assert_array_equal(host(s), rs)


def test_group_quant_empty():
    q, s = _ops().per_token_group_quant_int8(torch.empty((0, 128), device="cuda", dtype=torch.bfloat16), 64, 1e-6)
    assert q.shape == (0, 128) and s.shape == (0, 2)


@pytest.mark.parametrize("dt", ["FP32", "FP16", "BF16"])
@pytest.mark.parametrize("dims", [[8192, 4096], [1, 1024], [2, 16, 1024, 256], [333], [7, 13]])
def test_dynamic_quant_shapes(dt, dims):
    rng = seeded(len(dims) * 11 + dims[0])
    x = rng.standard_normal(dims).astype(np.float32)
    xt = dev(x, TORCH_DT[dt])
    x = host(xt).astype(np.float32)
    q, s, azp = _ops().dynamic_scaled_int8_quant(xt)
    rq, rs, _ = quant.dynamic_scaled_int8_quant(x, dt)
    np.testing.assert_array_equal(host(s), rs)
    np.testing.assert_array_equal(host(q), rq)


def test_dynamic_quant_all_zero_uses_min_scale():
    q, s, _ = _ops().dynamic_scaled_int8_quant(torch.zeros((4, 64), device="cuda"))
    assert host(s)[0] == np.float32(1.0 / (448.0 * 512.0))
    assert not host(q).any()


def test_repeat_calls_are_deterministic():
    x = dev(bf16_normal(seeded(9), (512, 4096)), torch.bfloat16)
    a = _ops().per_token_group_quant_int8(x, 128, 1e-6)
    b = _ops().per_token_group_quant_int8(x, 128, 1e-6)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
    c = _ops().dynamic_scaled_int8_quant(x)
    d = _ops().dynamic_scaled_int8_quant(x)
    assert torch.equal(c[0], d[0]) and torch.equal(c[1], d[1])


def _edge_rows(k):
    """FP32 rows that exercise the quotient edge cases of the fast quantiser path:
    row 0  amax 127 (scale exactly 1): ties k + 0.5 must round half to even;
    row 1  amax 1: values far below the FMA-division threshold (tiny normals, subnormals,
           signed zeros) next to ordinary ones;
    row 2  amax 1e-30 with a subnormal eps: a tiny but in-range scale;
    row 3  amax 1e-37: a scale below 2^-120, which takes the checked path."""
    rng = seeded(k)
    x = np.zeros((4, k), np.float32)
    ties = np.arange(-126, 127, dtype=np.float32) + np.float32(0.5)
    x[0] = rng.choice(ties, k)
    x[0, 0] = 127.0
    tiny = np.array([1e-30, -1e-30, 1e-38, -1e-38, 1e-40, -1e-40, 1e-45, -1e-45, 0.0, -0.0], np.float32)
    x[1] = np.where(rng.random(k) < 0.5, rng.choice(tiny, k), rng.standard_normal(k).astype(np.float32) * 0.3)
    x[1, 0] = 1.0
    x[2] = (rng.standard_normal(k) * 1e-31).astype(np.float32)
    x[2, 0] = 1e-30
    x[3] = (rng.standard_normal(k) * 1e-38).astype(np.float32)
    x[3, 0] = 1e-37
    return x


@pytest.mark.parametrize("g", [128, 4096])
def test_group_quant_ties_and_tiny_values(g):
    """Bit-exact codes where the quotient is a tie, far below the division threshold, or the
    scale itself is tiny (a subnormal eps lets the scale follow the amax) -- the subwarp
    (g = 128) and row-block (g = 4096) kernels."""
    x = _edge_rows(4096)
    eps = float(np.float32(1e-44))
    q, s = _ops().per_token_group_quant_int8(dev(x, torch.float32), g, eps)
    rq, rs = quant.per_token_group_quant_int8(x, g, eps)
    np.testing.assert_array_equal(host(s), rs)
    np.testing.assert_array_equal(host(q), rq)


def test_dynamic_quant_ties_and_tiny_values():
    x = _edge_rows(1024)[:2]                   # per-tensor: amax 127, so scale is exactly 1
    q, s, _ = _ops().dynamic_scaled_int8_quant(dev(x, torch.float32))
    rq, rs, _ = quant.dynamic_scaled_int8_quant(x, "FP32")
    np.testing.assert_array_equal(host(s), rs)
    np.testing.assert_array_equal(host(q), rq)


@pytest.mark.parametrize("name", golden_names("static_scaled_int8_quant"))
def test_static_quant_golden(name):
    meta, g = load_golden(name)
    x, xdt = g["x"]
    q = _ops().static_scaled_int8_quant(dev(x, TORCH_DT[xdt]), dev(g["scale"][0]), dev(g["azp"][0]))
    np.testing.assert_array_equal(host(q), g["q"][0])


@pytest.mark.parametrize("dt", ["FP32", "FP16", "BF16"])
@pytest.mark.parametrize("dims,scale,azp", [([512, 4096], 0.125, 0), ([7, 13], 0.02, 5), ([3, 1000], 1e-9, -7),
                                             ([2, 16, 1024], 3.0, 127), ([8191], 0.05, -128)])
def test_static_quant_shapes(dt, dims, scale, azp):
    """Odd sizes (scalar tail), a zero point, a scale below MIN_SCALE (clamped), ties and values far
    beyond +-127 * scale, against the oracle bit for bit."""
    rng = seeded(len(dims) * 5 + dims[0])
    x = (rng.standard_normal(dims) * 4).astype(np.float32)
    x.reshape(-1)[::97] = (np.arange(x.size)[::97] % 50 - 25 + 0.5) * np.float32(scale)   # exact ties
    xt = dev(x, TORCH_DT[dt])
    x = host(xt).astype(np.float32)
    s = dev(np.array([scale], np.float32))
    z = dev(np.array([azp], np.int32))
    q = _ops().static_scaled_int8_quant(xt, s, z)
    np.testing.assert_array_equal(host(q), quant.static_scaled_int8_quant(x, scale, azp))
