"""Pin the numpy oracle against fixtures produced by the reference's own Model.forward (CPU)."""
import numpy as np
import pytest

from conftest import golden_names, load_golden
from oracle import attention, gemm, kv_cache, numerics, quant, rmsnorm

DT = {"float32": "FP32", "float16": "FP16", "bfloat16": "BF16"}


@pytest.mark.parametrize("name", golden_names("dynamic_scaled_int8_quant"))
def test_dynamic_scaled_int8_quant(name):
    meta, g = load_golden(name)
    x, xdt = g["x"]
    q, s, azp = quant.dynamic_scaled_int8_quant(x, DT[xdt])
    np.testing.assert_array_equal(s, g["scale"][0])          # bit-exact scale
    np.testing.assert_array_equal(q, g["q"][0])              # bit-exact codes
    assert q.shape == g["q"][0].shape
    np.testing.assert_array_equal(azp, g["azp"][0])


@pytest.mark.parametrize("name", golden_names("per_token_group_quant_int8"))
def test_per_token_group_quant_int8(name):
    meta, g = load_golden(name)
    q, s = quant.per_token_group_quant_int8(g["x"][0], meta["group_size"], meta["eps"])
    np.testing.assert_array_equal(s, g["scales"][0])
    np.testing.assert_array_equal(q, g["q"][0])


@pytest.mark.parametrize("name", golden_names("add_rmsnorm"))
def test_add_rmsnorm(name):
    if name.startswith("add_rmsnorm_fp8"):
        pytest.skip("covered by test_add_rmsnorm_fp8")
    meta, g = load_golden(name)
    y = rmsnorm.add_rmsnorm(g["x"][0], g["residual"][0], g["weight"][0], meta["eps"], meta["dtype"])
    ref = g["out"][0].astype(np.float32)
    # reference reduces in float32 in its own order: allow a final-rounding step in the output dtype
    tol = {"FP32": 2e-6, "FP16": 1e-3, "BF16": 8e-3}[meta["dtype"]]
    np.testing.assert_allclose(y, ref, rtol=tol, atol=tol)
    if meta["dtype"] != "FP32":   # a 1-ulp float32 rsqrt difference rarely survives the final rounding
        assert np.mean(y == ref) > 0.97


@pytest.mark.parametrize("name", golden_names("add_rmsnorm_fp8"))
def test_add_rmsnorm_fp8(name):
    meta, g = load_golden(name)
    r_out, codes, scales, y = rmsnorm.add_rmsnorm_quant(g["x"][0], g["residual"][0], g["weight"][0], meta["eps"], "e4m3")
    np.testing.assert_array_equal(r_out, g["residual_out"][0])
    np.testing.assert_allclose(y, g["y"][0], rtol=2e-6, atol=2e-6)
    np.testing.assert_allclose(scales, g["scales"][0], rtol=2e-6)
    # one e4m3 ulp where y sits on a rounding boundary; almost all codes exact
    d = np.abs(numerics.e4m3_ordinal(codes) - numerics.e4m3_ordinal(g["codes"][0]))
    assert d.max() <= 1 and np.mean(d == 0) > 0.999


@pytest.mark.parametrize("name", golden_names("int8_scaled_mm_azp"))
def test_int8_scaled_mm_azp(name):
    meta, g = load_golden(name)
    ins = [g[k][0] for k in ("a", "b", "a_scales", "b_scales", "azp_adj", "azp", "bias")]
    out = gemm.int8_scaled_mm_azp(*ins, meta["has_azp"], meta["has_bias"], meta["output_dtype"])
    ref = g["out"][0].astype(np.float32)
    tol = {"FP32": 1e-5, "FP16": 2e-3, "BF16": 1e-2}[meta["output_dtype"]]
    np.testing.assert_allclose(out, ref, rtol=tol, atol=tol)


@pytest.mark.parametrize("name", golden_names("w8a8"))
def test_w8a8(name):
    meta, g = load_golden(name)
    acc = gemm.w8a8_acc(g["a"][0], g["b"][0])
    np.testing.assert_array_equal(acc, g["acc"][0])          # exact int32 accumulators
    out = gemm.w8a8_scaled_mm(g["a"][0], g["b"][0], g["sa"][0], g["sb"][0], g["bias"][0], "BF16", acc=acc)
    np.testing.assert_array_equal(out, g["out"][0])          # bit-exact bf16 epilogue


@pytest.mark.parametrize("name", golden_names("paged_kv_cache_update"))
def test_paged_kv_cache_update(name):
    meta, g = load_golden(name)
    out = kv_cache.paged_kv_cache_update(g["to_cache"][0], g["kv_cache"][0], g["slot_mapping"][0])
    np.testing.assert_array_equal(out, g["out"][0])


@pytest.mark.parametrize("name", golden_names("paged_attention"))
def test_paged_attention(name):
    meta, g = load_golden(name)
    args = [g[k][0] for k in ("query", "key_cache", "value_cache", "seq_lens", "block_table")]
    scale = meta["head_dim"] ** -0.5
    tol = {"FP32": 1e-5, "FP16": 2e-3, "BF16": 1e-2}[meta["output_dtype"]]
    o1 = attention.paged_attention_v1(*args, scale)
    np.testing.assert_allclose(o1, g["out_v1"][0].astype(np.float32), rtol=tol, atol=tol)
    o2, es, ml, tmp = attention.paged_attention_v2(*args, scale, meta["partition_size"])
    np.testing.assert_allclose(o2, g["out_v2"][0].astype(np.float32), rtol=tol, atol=tol)
    np.testing.assert_allclose(es, g["exp_sums"][0].astype(np.float32), rtol=tol, atol=tol)
    np.testing.assert_allclose(ml, g["max_logits"][0].astype(np.float32), rtol=tol, atol=tol)
    np.testing.assert_allclose(tmp, g["tmp_out"][0].astype(np.float32), rtol=tol, atol=tol)


@pytest.mark.parametrize("name", golden_names("batched_decode_attention"))
def test_batched_decode_attention(name):
    meta, g = load_golden(name)
    out = attention.batched_decode_attention(g["q"][0], g["k_cache"][0], g["v_cache"][0], g["seq_lens"][0],
                                             meta["head_dim"] ** -0.5)
    tol = {"FP32": 1e-5, "FP16": 2e-3, "BF16": 1e-2}[meta["dtype"]]
    np.testing.assert_allclose(out, g["out"][0].astype(np.float32), rtol=tol, atol=tol)


@pytest.mark.parametrize("name", golden_names("paged_fp8_decode"))
def test_paged_fp8_decode(name):
    meta, g = load_golden(name)
    kc = kv_cache.paged_fp8_kv_write(g["k_new"][0], g["k_cache"][0], g["slot_mapping"][0], g["k_scale"][0])
    vc = kv_cache.paged_fp8_kv_write(g["v_new"][0], g["v_cache"][0], g["slot_mapping"][0], g["v_scale"][0])
    np.testing.assert_array_equal(kc, g["k_cache_after"][0])
    np.testing.assert_array_equal(vc, g["v_cache_after"][0])
    slots = kv_cache.decode_slots(g["seq_lens"][0], g["block_table"][0], meta["block_size"])
    np.testing.assert_array_equal(slots, g["slot_mapping"][0])
    out = attention.paged_fp8_decode(g["query"][0], kc, vc, g["k_scale"][0], g["v_scale"][0], g["seq_lens"][0],
                                     g["block_table"][0], meta["head_dim"] ** -0.5)
    np.testing.assert_allclose(out, g["out"][0], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("name", golden_names("static_scaled_int8_quant"))
def test_static_scaled_int8_quant(name):
    meta, g = load_golden(name)
    q = quant.static_scaled_int8_quant(g["x"][0], g["scale"][0], g["azp"][0])
    np.testing.assert_array_equal(q, g["q"][0])              # bit-exact codes


@pytest.mark.parametrize("name", golden_names("kv_cache_write"))
def test_kv_cache_write(name):
    meta, g = load_golden(name)
    ko, vo = kv_cache.kv_cache_write(g["key_cache"][0], g["value_cache"][0], g["key"][0], g["value"][0],
                                     g["positions"][0])
    np.testing.assert_array_equal(ko, g["key_out"][0])
    np.testing.assert_array_equal(vo, g["value_out"][0])


@pytest.mark.parametrize("name", golden_names("flash_decoding_attention"))
def test_flash_decoding_attention(name):
    meta, g = load_golden(name)
    d = meta["head_dim"]
    out, es, ml, po = attention.flash_decoding_attention(g["query"][0], g["key_cache"][0], g["value_cache"][0],
                                                         meta["chunk_size"], meta["causal"], d ** -0.5)
    # the reference computes in float32 and rounds to the output dtype; the oracle in float64
    tol = {"FP32": 2e-5, "FP16": 2e-3, "BF16": 1.6e-2}[meta["dtype"]]
    np.testing.assert_allclose(out, g["out"][0], rtol=tol, atol=tol)
    np.testing.assert_allclose(po, g["partial_out"][0], rtol=tol, atol=tol)
    np.testing.assert_allclose(es, g["exp_sums"][0], rtol=tol, atol=tol)
    ref_ml = g["max_logits"][0]
    assert np.array_equal(np.isinf(ml), np.isinf(ref_ml))      # fully masked chunks: -inf
    fin = np.isfinite(ref_ml)
    np.testing.assert_allclose(ml[fin], ref_ml[fin], rtol=tol, atol=tol)


@pytest.mark.parametrize("name", golden_names("w8a8_act"))
def test_w8a8_act(name):
    meta, g = load_golden(name)
    out = gemm.w8a8_scaled_mm_act(g["a"][0], g["b_first"][0], g["b_second"][0], g["sa"][0], g["s_first"][0],
                                  g["s_second"][0], g["bias_first"][0], g["bias_second"][0], meta["act"], "BF16")
    ref = g["out"][0]
    # numpy's and torch's float32 exp may differ in the last bit, which can move a bf16 rounding
    np.testing.assert_allclose(out, ref, rtol=8e-3, atol=1e-6)
    assert np.mean(out == ref) > 0.99


@pytest.mark.parametrize("name", golden_names("flash_attn_with_kvcache"))
def test_flash_attn_with_kvcache(name):
    meta, g = load_golden(name)
    out, lse = attention.flash_attn_with_kvcache(g["q"][0], g["k_cache"][0], g["v_cache"][0], g["cache_seqlens"][0],
                                                 meta["head_dim"] ** -0.5)
    tol = {"FP32": 2e-5, "FP16": 2e-3, "BF16": 1.6e-2}[meta["dtype"]]
    np.testing.assert_allclose(out, g["out"][0], rtol=tol, atol=tol)
    np.testing.assert_allclose(lse, g["softmax_lse"][0], rtol=2e-5, atol=2e-5)


@pytest.mark.parametrize("name", golden_names("batched_prefill_attention"))
def test_batched_prefill_attention(name):
    meta, g = load_golden(name)
    out = attention.batched_prefill_attention(g["q"][0], g["k"][0], g["v"][0], g["qo_indptr"][0], g["kv_indptr"][0],
                                              meta["num_q_heads"], meta["num_kv_heads"], meta["head_dim"] ** -0.5)
    tol = {"FP32": 2e-5, "FP16": 2e-3, "BF16": 1.6e-2}[meta["dtype"]]
    np.testing.assert_allclose(out, g["out"][0], rtol=tol, atol=tol)
