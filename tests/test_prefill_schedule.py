"""CPU check of the tiled online softmax the prefill kernels use (no GPU).

The tcgen05 prefill kernel walks the keys in tiles of 128, keeps each row's max in the log2
domain but moves it only when a tile's max exceeds it by more than 2^8 (otherwise it keeps
exponentiating against the stale max), rounds P to the 16-bit input type for the P.V product
while summing the unrounded P, and divides by the sum at the end.  This restates that schedule
in numpy and checks it against the float64 softmax of the oracle: the lazy max must not change
the result beyond the rounding of P, including when the scores drift upwards so that the
max moves several times, and when the first tiles are far below the later ones.
"""
import numpy as np
import pytest

from oracle import attention
from oracle.numerics import round_bf16


def _tiled(q, k, v, scale, lazy, tile=128):
    """One head, causal with q_len == kv_len: the kernel's per-row schedule in float32."""
    n, d = q.shape
    c = np.float32(scale * np.log2(np.e))
    m = np.full(n, -np.inf, np.float32)
    l = np.zeros(n, np.float32)
    o = np.zeros((n, d), np.float32)
    s_all = (q.astype(np.float32) @ k.astype(np.float32).T).astype(np.float32)
    for j0 in range(0, n, tile):
        s = s_all[:, j0:j0 + tile].copy()
        keys = np.arange(j0, min(j0 + tile, n))
        s[keys[None, :] > np.arange(n)[:, None]] = -np.inf
        mx = s.max(axis=1) * c
        grow = mx > m + (lazy if lazy else 0.0)
        alpha = np.where(grow, np.exp2(m - mx), np.float32(1.0)).astype(np.float32)
        m = np.where(grow, mx, m).astype(np.float32)
        p = np.exp2(s * c - m[:, None]).astype(np.float32)
        l = (l * alpha + p.sum(axis=1)).astype(np.float32)
        o = (o * alpha[:, None] + round_bf16(p) @ v[j0:j0 + tile].astype(np.float32)).astype(np.float32)
    return o / l[:, None]


@pytest.mark.parametrize("drift", [0.0, 0.02, 0.2])
def test_lazy_rescale_matches_softmax(drift):
    rng = np.random.default_rng(7)
    n, d = 640, 64
    q = round_bf16(rng.standard_normal((n, d)).astype(np.float32))
    k = round_bf16((rng.standard_normal((n, d)) + drift * np.arange(n)[:, None] / 8).astype(np.float32))
    v = round_bf16(rng.standard_normal((n, d)).astype(np.float32))
    ind = np.array([0, n], np.int32)
    ref = attention.batched_prefill_attention(q[:, None], k[:, None], v[:, None], ind, ind, 1, 1, d ** -0.5)[:, 0]
    lazy = _tiled(q, k, v, d ** -0.5, lazy=8.0)
    eager = _tiled(q, k, v, d ** -0.5, lazy=0.0)
    # the reference's bf16 tolerance, and the lazy and eager schedules agree to P's rounding
    np.testing.assert_allclose(lazy, ref, rtol=1.5e-2, atol=1e-2)
    np.testing.assert_allclose(lazy, eager, rtol=1e-2, atol=4e-3)
    assert np.mean(np.abs(lazy - ref)) <= 2e-3
