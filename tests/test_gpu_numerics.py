"""The kernels' FMA-corrected (Markstein) division must equal IEEE float32 division bit for bit.

Every quantisation kernel computes x / scale as div_rn(x, make_divisor(scale)); the int8
and e4m3 codes are only bit-exact against the reference if this equals numpy's (IEEE)
float32 quotient for every input of its domain, |a| <= 2^100 * b (the quantisers always
have |a| <= 448 * b), including signed zeros, tiny and huge operands, divisors outside
[2^-120, 2^120] and quotients next to rounding midpoints.
"""
import numpy as np
import pytest
import torch

from gpu_util import require_gpu

pytestmark = pytest.mark.gpu


def _run(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    from kernelverse_b200 import _lib
    at, bt = torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()
    out = torch.empty_like(at)
    _lib.call("kvb_selftest_div_rn", at.data_ptr(), bt.data_ptr(), out.data_ptr(), a.size,
              torch.cuda.current_stream().cuda_stream)
    return out.cpu().numpy()


def _in_domain(a, b):
    keep = np.abs(a).astype(np.float64) <= np.exp2(100.0) * b.astype(np.float64)
    return a[keep], b[keep]


def _assert_same_bits(got, a, b):
    want = (a / b).astype(np.float32)
    g, w = got.view(np.uint32), want.view(np.uint32)
    both_nan = np.isnan(got) & np.isnan(want)
    bad = (g != w) & ~both_nan
    assert not bad.any(), f"{bad.sum()} mismatches, first a={a[bad][0]!r} b={b[bad][0]!r} got={got[bad][0]!r} want={want[bad][0]!r}"


def test_div_random_binades():
    require_gpu()
    rng = np.random.default_rng(0)
    n = 1 << 24
    a = (rng.standard_normal(n) * np.exp2(rng.integers(-130, 127, n))).astype(np.float32)
    b = np.abs(rng.standard_normal(n) * np.exp2(rng.integers(-40, 40, n))).astype(np.float32) + np.float32(1e-30)
    a, b = _in_domain(a, b)
    assert a.size > n // 2
    _assert_same_bits(_run(a, b), a, b)


def test_div_quantisation_ranges():
    """Divisors of the form amax/127 and amax/448, dividends within +-amax (the kernels' use)."""
    require_gpu()
    rng = np.random.default_rng(1)
    n = 1 << 24
    amax = np.abs(rng.standard_normal(n).astype(np.float32) * 10) + np.float32(1e-3)
    b = np.where(rng.random(n) < 0.5, amax / np.float32(127), amax / np.float32(448)).astype(np.float32)
    a = (amax * (rng.random(n) * 2 - 1)).astype(np.float32)
    _assert_same_bits(_run(a, b), a, b)


def test_div_near_midpoints_and_specials():
    require_gpu()
    rng = np.random.default_rng(2)
    n = 1 << 22
    b = (rng.random(n) * 8 + 1e-3).astype(np.float32)
    q = (rng.standard_normal(n) * 100).astype(np.float32)
    mid = q.astype(np.float64) + np.spacing(q).astype(np.float64) / 2           # exact midpoints of float32 quotients
    a = (mid * b.astype(np.float64)).astype(np.float32)                          # a/b within an ulp of a midpoint
    specials_a = np.array([0.0, -0.0, 1e-40, -1e-40, 1e-30, 3.4e38, -3.4e38, 1.0, -1.0, 127.0, 448.0, 2e-30],
                          np.float32)
    specials_b = np.array([1.0, 1.0, 1e-6, 3.0, 7.0, 2.0 ** 100, 2.0 ** 120, 2.0 ** -125, 2.0 ** 125, 1e-6, 1e-38,
                           2.0 ** 90], np.float32)
    a = np.concatenate([a, specials_a, np.nextafter(a[:100000], np.float32(np.inf))])
    b = np.concatenate([b, specials_b, b[:100000]])
    a, b = _in_domain(a, b)
    _assert_same_bits(_run(a, b), a, b)


def test_all_mantissas_of_one_binade():
    """Every float32 in [1, 2) divided by a few awkward divisors."""
    require_gpu()
    a = (np.arange(1 << 23, dtype=np.uint32) | np.uint32(0x3F800000)).view(np.float32)
    for bv in (np.float32(3.0), np.float32(np.nextafter(np.float32(2.0), np.float32(0))), np.float32(1.0 / 127),
               np.float32(0.7071068), np.float32(448.0 / 127)):
        b = np.full_like(a, bv)
        _assert_same_bits(_run(a, b), a, b)
