"""Known-answer tests for the oracle's bf16 and e4m3fn helpers (CPU).

The e4m3fn expectations come from the format definition (OCP FP8 E4M3: bias 7,
3 mantissa bits, max finite 448 = 1.75 * 2**8, subnormals m * 2**-9, no
infinities, NaN = S.1111.111) and from torch's own ``float8_e4m3fn`` cast.
"""
import numpy as np
import torch

from oracle import numerics as nm


def test_e4m3_known_answers():
    cases = {
        0.0: 0x00, 448.0: 0x7E, -448.0: 0xFE, 1.0: 0x38, -1.0: 0xB8, 2.0 ** -6: 0x08,   # min normal
        2.0 ** -9: 0x01, 7 * 2.0 ** -9: 0x07,                                             # subnormals
        2.0 ** -10: 0x00, 3 * 2.0 ** -10: 0x02, 5 * 2.0 ** -10: 0x02,                   # RNE ties
        1.0625: 0x38, 1.1875: 0x3A, 416.0: 0x7D, 440.0: 0x7E, 1.5: 0x3C, 240.0: 0x77,
    }
    xs = np.array(list(cases.keys()), np.float32)
    np.testing.assert_array_equal(nm.e4m3_encode(xs), np.array(list(cases.values()), np.uint8))


def test_e4m3_roundtrip_all_codes():
    codes = np.arange(256, dtype=np.uint8)
    finite = (codes & 0x7F) != 0x7F
    vals = nm.e4m3_decode(codes)
    assert np.all(np.isnan(vals[~finite]))
    back = nm.e4m3_encode(vals[finite])
    # -0.0 decodes to -0 and encodes back to 0x80
    np.testing.assert_array_equal(back, codes[finite])
    tv = torch.from_numpy(codes.copy()).view(torch.float8_e4m3fn).float().numpy()
    np.testing.assert_array_equal(vals[finite], tv[finite])


def test_e4m3_matches_torch_cast_on_midpoints_and_random():
    vals = nm.e4m3_decode(np.arange(0, 0x7F, dtype=np.uint8)).astype(np.float64)
    mids = (vals[:-1] + vals[1:]) / 2
    rng = np.random.default_rng(0)
    xs = np.concatenate([mids, np.nextafter(mids, 0), np.nextafter(mids, 1e9),
                         rng.standard_normal(20000) * 50, rng.standard_normal(5000) * 1e-3])
    xs = np.clip(np.concatenate([xs, -xs]), -448, 448).astype(np.float32)
    ours = nm.e4m3_encode(xs)
    theirs = torch.from_numpy(xs).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    np.testing.assert_array_equal(ours, theirs)


def test_bf16_rounding_matches_torch():
    rng = np.random.default_rng(1)
    xs = np.concatenate([rng.standard_normal(50000).astype(np.float32) * 10,
                         (np.arange(1 << 16, dtype=np.uint32) << 16 | 0x8000).view(np.float32)[:60000]])
    xs = xs[np.isfinite(xs)]
    theirs = torch.from_numpy(xs).to(torch.bfloat16).float().numpy()
    np.testing.assert_array_equal(nm.round_bf16(xs), theirs)


def test_e4m3_ordinal_counts_ulps():
    a = np.array([0x38, 0x39, 0xB8, 0x00, 0x80], np.uint8)
    o = nm.e4m3_ordinal(a)
    assert o[1] - o[0] == 1 and o[0] == -o[2] and o[3] == o[4] == 0
