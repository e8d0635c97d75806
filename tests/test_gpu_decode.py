"""GPU parity of paged decode attention and the paged KV-cache writes against the oracle.

Tolerances: float32 caches are computed in float32 on CUDA cores (|err| <= 1e-5 + 1e-5 |ref|);
f16/bf16/e4m3 caches run QK^T and PV on tensor cores with f16 (bf16) probabilities and
float32 accumulation, then round to the output dtype: |err| <= 1e-2 + 1e-2 |ref| (the
BASELINE bf16 tolerance) with the mean error at most 1e-3.  Cache writes are bit-exact.
"""
import numpy as np
import pytest
import torch

from conftest import golden_names, load_golden
from gpu_util import TORCH_DT, dev, host, require_gpu, seeded
from oracle import attention, kv_cache, numerics

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _gpu():
    require_gpu()


def _ops():
    from kernelverse_b200 import ops
    return ops


def _close(got, ref, tight: bool):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    if tight:
        np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-5)
    else:
        np.testing.assert_allclose(got, ref, rtol=1e-2, atol=1e-2)
        assert np.mean(np.abs(got - ref)) <= 1e-3


@pytest.mark.parametrize("name", golden_names("paged_attention"))
def test_paged_attention_golden(name):
    meta, g = load_golden(name)
    dt = TORCH_DT[meta["input_dtype"]]
    kc, vc = g["key_cache"][0], g["value_cache"][0]
    nb, bs, hkv, d = kc.shape
    # the reference's declared shape [nb, Hkv, bs, D] over the same memory
    kt = dev(kc, dt).view(nb, hkv, bs, d)
    vt = dev(vc, dt).view(nb, hkv, bs, d)
    q = dev(g["query"][0], dt)
    sl = dev(g["seq_lens"][0])
    bt = dev(g["block_table"][0])
    tight = meta["input_dtype"] == "FP32"
    out = _ops().paged_attention_v1(q, kt, vt, sl, bt)
    assert out.dtype == dt
    _close(host(out), g["out_v1"][0], tight)
    out2, es, ml, tmp = _ops().paged_attention_v2(q, kt, vt, sl, bt, meta["partition_size"])
    assert tuple(es.shape) == g["exp_sums"][0].shape and tuple(tmp.shape) == g["tmp_out"][0].shape
    _close(host(out2), g["out_v2"][0], tight)
    _close(host(tmp), g["tmp_out"][0], tight)
    m_ref, m_got = g["max_logits"][0], host(ml)
    assert np.array_equal(np.isinf(m_ref), np.isinf(m_got))
    fin = np.isfinite(m_ref)
    np.testing.assert_allclose(m_got[fin], m_ref[fin], rtol=1e-2 if not tight else 1e-5, atol=1e-2 if not tight else 1e-5)
    np.testing.assert_allclose(host(es), g["exp_sums"][0], rtol=2e-2 if not tight else 1e-5, atol=1e-2 if not tight else 1e-5)


@pytest.mark.parametrize("name", golden_names("batched_decode_attention"))
def test_batched_decode_golden(name):
    meta, g = load_golden(name)
    dt = TORCH_DT[meta["dtype"]]
    out = _ops().batched_decode_attention(dev(g["q"][0], dt), dev(g["k_cache"][0], dt), dev(g["v_cache"][0], dt),
                                          dev(g["seq_lens"][0]))
    _close(host(out), g["out"][0], meta["dtype"] == "FP32")


@pytest.mark.parametrize("name", golden_names("paged_kv_cache_update"))
def test_kv_cache_update_golden(name):
    meta, g = load_golden(name)
    dt = TORCH_DT[meta["dtype"]]
    src = dev(g["kv_cache"][0], dt)
    out = _ops().paged_kv_cache_update(dev(g["to_cache"][0], dt), src, dev(g["slot_mapping"][0]))
    np.testing.assert_array_equal(host(out), g["out"][0].astype(np.float32))
    np.testing.assert_array_equal(host(src), g["kv_cache"][0].astype(np.float32))   # input untouched


@pytest.mark.parametrize("name", golden_names("paged_fp8_decode"))
def test_fp8_decode_golden(name):
    meta, g = load_golden(name)
    u8 = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda().view(torch.float8_e4m3fn)  # noqa: E731
    kc, vc = u8(g["k_cache"][0]), u8(g["v_cache"][0])
    out = _ops().paged_fp8_decode(dev(g["query"][0], torch.bfloat16), kc, vc, dev(g["k_scale"][0]), dev(g["v_scale"][0]),
                                  dev(g["seq_lens"][0]), dev(g["block_table"][0]),
                                  k_new=dev(g["k_new"][0], torch.bfloat16), v_new=dev(g["v_new"][0], torch.bfloat16))
    np.testing.assert_array_equal(host(kc), g["k_cache_after"][0])
    np.testing.assert_array_equal(host(vc), g["v_cache_after"][0])
    _close(host(out), g["out"][0], False)


def make_fp8_case(rng, B, hq, hkv, D, bs, lens, extra_blocks=3):
    maxb = max((L + bs - 1) // bs for L in lens)
    nblocks = sum((L + bs - 1) // bs for L in lens) + extra_blocks
    perm = rng.permutation(nblocks).astype(np.int32)
    bt = np.zeros((B, maxb), np.int32)
    pos = 0
    for b, L in enumerate(lens):
        nb = (L + bs - 1) // bs
        bt[b, :nb] = perm[pos:pos + nb]
        pos += nb
    k_scale = (rng.random(hkv) * 0.01 + 0.005).astype(np.float32)
    v_scale = (rng.random(hkv) * 0.01 + 0.005).astype(np.float32)
    kc = numerics.e4m3_quantize(rng.standard_normal((nblocks, bs, hkv, D)).astype(np.float32), k_scale[None, None, :, None])
    vc = numerics.e4m3_quantize(rng.standard_normal((nblocks, bs, hkv, D)).astype(np.float32), v_scale[None, None, :, None])
    q = numerics.round_bf16(rng.standard_normal((B, hq, D)).astype(np.float32))
    k_new = numerics.round_bf16(rng.standard_normal((B, hkv, D)).astype(np.float32))
    v_new = numerics.round_bf16(rng.standard_normal((B, hkv, D)).astype(np.float32))
    return dict(q=q, kc=kc, vc=vc, k_scale=k_scale, v_scale=v_scale, bt=bt, lens=np.array(lens, np.int32),
                k_new=k_new, v_new=v_new)


def run_fp8(case, fused=True, partition_size=0):
    u8 = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda().view(torch.float8_e4m3fn)  # noqa: E731
    kc, vc = u8(case["kc"]), u8(case["vc"])
    out = _ops().paged_fp8_decode(dev(case["q"], torch.bfloat16), kc, vc, dev(case["k_scale"]), dev(case["v_scale"]),
                                  dev(case["lens"]), dev(case["bt"]),
                                  k_new=dev(case["k_new"], torch.bfloat16) if fused else None,
                                  v_new=dev(case["v_new"], torch.bfloat16) if fused else None,
                                  partition_size=partition_size)
    return out, kc, vc


def oracle_fp8(case, fused=True):
    bs = case["kc"].shape[1]
    kc, vc = case["kc"], case["vc"]
    if fused:
        slots = kv_cache.decode_slots(case["lens"], case["bt"], bs)
        kc = kv_cache.paged_fp8_kv_write(case["k_new"], kc, slots, case["k_scale"])
        vc = kv_cache.paged_fp8_kv_write(case["v_new"], vc, slots, case["v_scale"])
    D = kc.shape[-1]
    out = attention.paged_fp8_decode(case["q"], kc, vc, case["k_scale"], case["v_scale"], case["lens"], case["bt"], D ** -0.5)
    return out, kc, vc


@pytest.mark.parametrize("B,hq,hkv,D,bs,lens,part", [
    (4, 32, 8, 128, 16, [1, 17, 300, 1000], 0),
    (3, 8, 1, 128, 16, [513, 48, 16], 256),
    (2, 16, 16, 64, 32, [100, 33], 64),
    (3, 16, 2, 128, 8, [40, 7, 1], 0),
    (2, 32, 2, 64, 16, [2000, 1], 512),
    (2, 32, 1, 128, 1, [20, 5], 0),
    # more (kv head, 8-query) tiles than 16 warps: KV heads split over CTAs
    (2, 64, 32, 128, 16, [300, 77], 0),
    (1, 256, 8, 64, 16, [70], 128),
])
def test_fp8_decode_shapes(B, hq, hkv, D, bs, lens, part):
    case = make_fp8_case(seeded(B * 100 + hq + D + bs), B, hq, hkv, D, bs, lens)
    out, kc, vc = run_fp8(case, True, part)
    ref, rk, rv = oracle_fp8(case, True)
    np.testing.assert_array_equal(host(kc), rk)
    np.testing.assert_array_equal(host(vc), rv)
    _close(host(out), ref, False)


def test_fp8_decode_baseline_config_full_size():
    """BASELINE fourth config: B=64, 32/8 heads, D=128, bs=16, ctx ~ U[512, 8192], permuted blocks."""
    rng = seeded(4)
    lens = rng.integers(512, 8193, 64).tolist()
    case = make_fp8_case(rng, 64, 32, 8, 128, 16, lens)
    out, kc, vc = run_fp8(case, True)
    ref, rk, rv = oracle_fp8(case, True)
    np.testing.assert_array_equal(host(kc), rk)
    np.testing.assert_array_equal(host(vc), rv)
    _close(host(out), ref, False)
    # determinism: a second call over the already-written cache gives identical results
    out2, _, _ = run_fp8(dict(case, kc=host(kc), vc=host(vc)), True)
    assert torch.equal(out, out2)


@pytest.mark.parametrize("dt", ["FP32", "FP16", "BF16"])
@pytest.mark.parametrize("B,hq,hkv,D,bs,lens,part", [
    (3, 32, 8, 128, 16, [700, 1, 64], 128),
    (2, 8, 1, 64, 32, [100, 257], 64),
    (2, 16, 4, 128, 4, [50, 3], 256),
])
def test_paged_attention_dtypes(dt, B, hq, hkv, D, bs, lens, part):
    rng = seeded(B + hq + D + bs)
    tdt = TORCH_DT[dt]
    case = make_fp8_case(rng, B, hq, hkv, D, bs, lens)
    kc = host(dev(rng.standard_normal(case["kc"].shape).astype(np.float32), tdt)).astype(np.float32)
    vc = host(dev(rng.standard_normal(case["vc"].shape).astype(np.float32), tdt)).astype(np.float32)
    q = host(dev(rng.standard_normal(case["q"].shape).astype(np.float32), tdt)).astype(np.float32)
    nb = kc.shape[0]
    kt = dev(kc, tdt).view(nb, hkv, bs, D)
    vt = dev(vc, tdt).view(nb, hkv, bs, D)
    out = _ops().paged_attention_v1(dev(q, tdt), kt, vt, dev(case["lens"]), dev(case["bt"]))
    ref = attention.paged_attention_v1(q, kc, vc, case["lens"], case["bt"], D ** -0.5)
    _close(host(out), ref, dt == "FP32")
    o2, es, ml, tmp = _ops().paged_attention_v2(dev(q, tdt), kt, vt, dev(case["lens"]), dev(case["bt"]), part)
    r2, res_, rml, rtmp = attention.paged_attention_v2(q, kc, vc, case["lens"], case["bt"], D ** -0.5, part)
    _close(host(o2), r2, dt == "FP32")
    _close(host(tmp), rtmp, dt == "FP32")


def test_fp8_kv_write_standalone():
    rng = seeded(11)
    nb, bs, hkv, D, T = 10, 16, 8, 128, 37
    cache = np.zeros((nb, bs, hkv, D), np.uint8)
    x = numerics.round_bf16(rng.standard_normal((T, hkv, D)).astype(np.float32))
    slots = rng.permutation(nb * bs)[:T].astype(np.int64)
    slots[::5] = -1
    sc = (rng.random(hkv) * 0.01 + 0.005).astype(np.float32)
    ct = torch.from_numpy(cache.copy()).cuda().view(torch.float8_e4m3fn)
    _ops().paged_fp8_kv_write(dev(x, torch.bfloat16), ct, dev(slots), dev(sc))
    np.testing.assert_array_equal(host(ct), kv_cache.paged_fp8_kv_write(x, cache, slots, sc))


def test_kv_cache_update_large_and_int32():
    rng = seeded(12)
    nb, bs, h, d, T = 4096, 16, 16, 128, 8192
    cache = rng.standard_normal((nb, bs, h, d)).astype(np.float32)
    to = rng.standard_normal((T, h, d)).astype(np.float32)
    slots = rng.permutation(nb * bs)[:T].astype(np.int32)
    slots[::7] = -1
    out = _ops().paged_kv_cache_update(dev(to), dev(cache), dev(slots))
    np.testing.assert_array_equal(host(out), kv_cache.paged_kv_cache_update(to, cache, slots))


@pytest.mark.parametrize("name", golden_names("kv_cache_write"))
def test_kv_cache_write_golden(name):
    meta, g = load_golden(name)
    dt = {"FP32": torch.float32, "FP16": torch.float16, "BF16": torch.bfloat16}[meta["dtype"]]
    ko, vo = _ops().kv_cache_write(dev(g["key_cache"][0], dt), dev(g["value_cache"][0], dt), dev(g["key"][0], dt),
                                   dev(g["value"][0], dt), dev(g["positions"][0]))
    np.testing.assert_array_equal(host(ko), g["key_out"][0].astype(np.float32) if dt != torch.float32 else g["key_out"][0])
    np.testing.assert_array_equal(host(vo), g["value_out"][0].astype(np.float32) if dt != torch.float32 else g["value_out"][0])


@pytest.mark.parametrize("per_batch", [False, True])
def test_kv_cache_write_large_and_negative_positions(per_batch):
    """A prefill-sized write (16 heads x 512 rows) with int32 positions, negative ones counting
    from the end as torch indexing does; inputs stay untouched."""
    rng = seeded(31)
    b, h, s, w, d = 4, 16, 2048, 512, 128
    kc = rng.standard_normal((b, h, s, d)).astype(np.float32)
    vc = rng.standard_normal((b, h, s, d)).astype(np.float32)
    k = rng.standard_normal((b, h, w, d)).astype(np.float32)
    v = rng.standard_normal((b, h, w, d)).astype(np.float32)
    if per_batch:
        pos = np.stack([np.arange(w) + 100 * i for i in range(b)]).astype(np.int32)
        pos[:, -3:] -= s                                      # the last three as negative indices
    else:
        pos = (np.arange(w) + 1000).astype(np.int32)
        pos[:5] = pos[:5] - s
    bf = torch.bfloat16
    kct, vct = dev(kc, bf), dev(vc, bf)
    keep = kct.clone()
    ko, vo = _ops().kv_cache_write(kct, vct, dev(k, bf), dev(v, bf), dev(pos))
    rk, rv = kv_cache.kv_cache_write(host(kct), host(vct), host(dev(k, bf)), host(dev(v, bf)), pos)
    np.testing.assert_array_equal(host(ko), rk)
    np.testing.assert_array_equal(host(vo), rv)
    assert torch.equal(kct, keep)


@pytest.mark.parametrize("name", golden_names("flash_decoding_attention"))
def test_flash_decoding_golden(name):
    meta, g = load_golden(name)
    dt = {"FP32": torch.float32, "FP16": torch.float16, "BF16": torch.bfloat16}[meta["dtype"]]
    out, es, ml, po = _ops().flash_decoding_attention(dev(g["query"][0], dt), dev(g["key_cache"][0], dt),
                                                      dev(g["value_cache"][0], dt), meta["chunk_size"], meta["causal"])
    tight = dt == torch.float32
    tol = 5e-4 if tight else (1e-2 if dt == torch.float16 else 1.5e-2)   # the reference's config.json tolerances
    for got, ref in ((out, g["out"][0]), (po, g["partial_out"][0]), (es, g["exp_sums"][0])):
        np.testing.assert_allclose(host(got), ref.astype(np.float32), rtol=tol, atol=tol)
    ref_ml = g["max_logits"][0].astype(np.float32)
    got_ml = host(ml)
    assert np.array_equal(np.isneginf(got_ml), np.isneginf(ref_ml))
    fin = np.isfinite(ref_ml)
    np.testing.assert_allclose(got_ml[fin], ref_ml[fin], rtol=tol, atol=tol)


@pytest.mark.parametrize("dt", ["FP32", "BF16"])
@pytest.mark.parametrize("b,sq,s,h,d,chunk,causal", [(4, 1, 2048, 16, 128, 256, False), (2, 16, 2048, 8, 64, 256, True),
                                                     (1, 64, 1024, 4, 128, 128, True), (2, 8, 520, 3, 64, 64, False)])
def test_flash_decoding_shapes(dt, b, sq, s, h, d, chunk, causal):
    rng = seeded(b * 100 + sq)
    q = rng.standard_normal((b, h, sq, d)).astype(np.float32)
    k = rng.standard_normal((b, h, s, d)).astype(np.float32)
    v = rng.standard_normal((b, h, s, d)).astype(np.float32)
    tdt = TORCH_DT[dt]
    qt, kt, vt = dev(q, tdt), dev(k, tdt), dev(v, tdt)
    out, es, ml, po = _ops().flash_decoding_attention(qt, kt, vt, chunk, causal)
    r_out, r_es, r_ml, r_po = attention.flash_decoding_attention(host(qt), host(kt), host(vt), chunk, causal, d ** -0.5)
    tight = dt == "FP32"
    _close(host(out), r_out, tight)
    _close(host(po), r_po, tight)
    np.testing.assert_allclose(host(es), r_es, rtol=1e-5 if tight else 1e-2, atol=1e-5 if tight else 1e-2)
    assert np.array_equal(np.isneginf(host(ml)), np.isneginf(r_ml))


@pytest.mark.parametrize("name", golden_names("flash_attn_with_kvcache"))
def test_flash_attn_with_kvcache_golden(name):
    meta, g = load_golden(name)
    dt = {"FP32": torch.float32, "FP16": torch.float16, "BF16": torch.bfloat16}[meta["dtype"]]
    out, lse = _ops().flash_attn_with_kvcache(dev(g["q"][0], dt), dev(g["k_cache"][0], dt), dev(g["v_cache"][0], dt),
                                              dev(g["cache_seqlens"][0]))
    tol = 5e-4 if dt == torch.float32 else (1e-2 if dt == torch.float16 else 1.5e-2)   # config.json
    np.testing.assert_allclose(host(out), g["out"][0].astype(np.float32), rtol=tol, atol=tol)
    np.testing.assert_allclose(host(lse), g["softmax_lse"][0], rtol=1e-4 if dt == torch.float32 else 2e-3,
                               atol=1e-4 if dt == torch.float32 else 2e-3)


@pytest.mark.parametrize("dt", ["FP32", "BF16", "FP16"])
@pytest.mark.parametrize("b,sq,sk,h,hkv,d,ragged", [(4, 1, 2048, 16, 16, 128, False), (2, 16, 2048, 16, 16, 64, True),
                                                    (8, 1, 4096, 32, 32, 128, True), (2, 32, 1000, 32, 8, 128, False),
                                                    (3, 5, 333, 8, 2, 64, True), (2, 32, 700, 32, 4, 128, True),
                                                    (2, 24, 500, 24, 2, 64, True)])
def test_flash_attn_with_kvcache_shapes(dt, b, sq, sk, h, hkv, d, ragged):
    """Query tokens per sequence, ragged lengths, GQA, and 32 KV heads (split over CTAs).  The
    16-bit kernels fold a sequence's query tokens into one CTA row: all of them, or (group 8 x
    32 tokens, group 12 x 24 tokens) the largest divisor that fits, two or three CTA rows a
    sequence."""
    rng = seeded(b * 1000 + sq * 10 + h)
    q = rng.standard_normal((b, sq, h, d)).astype(np.float32)
    k = rng.standard_normal((b, sk, hkv, d)).astype(np.float32)
    v = rng.standard_normal((b, sk, hkv, d)).astype(np.float32)
    lens = (rng.integers(1, sk + 1, b) if ragged else np.full(b, sk)).astype(np.int32)
    tdt = TORCH_DT[dt]
    qt, kt, vt = dev(q, tdt), dev(k, tdt), dev(v, tdt)
    out, lse = _ops().flash_attn_with_kvcache(qt, kt, vt, dev(lens))
    r_out, r_lse = attention.flash_attn_with_kvcache(host(qt), host(kt), host(vt), lens, d ** -0.5)
    _close(host(out), r_out, dt == "FP32")
    np.testing.assert_allclose(host(lse), r_lse, rtol=1e-4, atol=1e-4 if dt == "FP32" else 2e-3)



def test_fp8_decode_partition_boundaries():
    """Rows whose lengths end exactly on, just before and just after partition boundaries (the
    last partition full, one row long, or one row short)."""
    lens = [512, 1024, 513, 511, 1, 1536, 2047, 16]
    case = make_fp8_case(seeded(31), len(lens), 32, 8, 128, 16, lens)
    out, kc, vc = run_fp8(case, True, 512)
    ref, rk, rv = oracle_fp8(case, True)
    np.testing.assert_array_equal(host(kc), rk)
    _close(host(out), ref, False)


def test_fp8_decode_many_rows_plain_grid():
    """1100 short rows (a grid of 1100 x 3 CTAs, most of them past their row's end)."""
    rng = seeded(32)
    lens = rng.integers(1, 40, 1100).tolist()
    case = make_fp8_case(rng, 1100, 8, 1, 128, 16, lens)
    out, kc, vc = run_fp8(case, True, 16)
    ref, rk, rv = oracle_fp8(case, True)
    np.testing.assert_array_equal(host(kc), rk)
    _close(host(out), ref, False)


def test_fp8_decode_repeated_calls_and_graph_replay():
    """Repeated calls and replays of one captured launch (decode + merge as programmatic
    dependents inside a CUDA graph) give the first call's result bit for bit."""
    rng = seeded(33)
    lens = rng.integers(100, 3000, 24).tolist()
    case = make_fp8_case(rng, 24, 32, 8, 128, 16, lens)
    bf = torch.bfloat16
    u8 = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda().view(torch.float8_e4m3fn)  # noqa: E731
    args = (dev(case["q"], bf), u8(case["kc"]), u8(case["vc"]), dev(case["k_scale"]), dev(case["v_scale"]),
            dev(case["lens"]), dev(case["bt"]))
    first = _ops().paged_fp8_decode(*args)
    ref, _, _ = oracle_fp8(case, False)
    _close(host(first), ref, False)
    for _ in range(70):
        assert torch.equal(_ops().paged_fp8_decode(*args), first)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        _ops().paged_fp8_decode(*args)          # warm-up on the capture stream
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        captured = _ops().paged_fp8_decode(*args)
    for _ in range(5):
        captured.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(captured, first)
