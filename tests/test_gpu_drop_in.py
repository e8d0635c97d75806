"""Each drop-in ModelNew file, executed the way KernelVerse's CudaBackend.compile executes
generated code (backends/cuda_backend.py:35-45), reproduces the reference Model's outputs
(golden fixtures) within the reference's own per-operator tolerances (config.json)."""
import numpy as np
import pytest
import torch

from conftest import golden_names, load_golden
from gpu_util import TORCH_DT, dev, host, require_gpu
from kernelverse_b200 import drop_in

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _gpu():
    require_gpu()


def modelnew(op, shape):
    ctx = {}
    exec(compile(drop_in.path(op).read_text(), str(drop_in.path(op)), "exec"), ctx)
    return ctx["ModelNew"](dict(shape, _baseline_compute_mode="performance")).cuda().eval()


def _as_dev(arr, dt):
    if dt in ("bfloat16", "float16", "float32"):
        return dev(arr, TORCH_DT[dt])
    return dev(arr)


def _check(got, ref, dtname, tol):
    g = host(got).astype(np.float64)
    r = np.asarray(ref, np.float64)
    if dtname in ("int8", "int32", "int64"):
        assert np.max(np.abs(g - r)) <= tol.get("max_abs_diff", 0)
    else:
        np.testing.assert_allclose(g, r, rtol=tol["rtol"], atol=tol["atol"])


TOL = {"FP32": {"rtol": 5e-4, "atol": 5e-4}, "FP16": {"rtol": 1e-2, "atol": 1e-2}, "BF16": {"rtol": 1.5e-2, "atol": 1e-2}}
DT = {"float32": "FP32", "float16": "FP16", "bfloat16": "BF16"}


@pytest.mark.parametrize("name", golden_names("dynamic_scaled_int8_quant"))
def test_dynamic_scaled_int8_quant(name):
    meta, g = load_golden(name)
    q, s, azp = modelnew("dynamic_scaled_int8_quant", meta)(_as_dev(*g["x"]))
    assert q.dtype == torch.int8 and tuple(q.shape) == g["q"][0].shape
    _check(q, g["q"][0], "int8", {"max_abs_diff": 0})
    _check(s, g["scale"][0], "float32", TOL["FP32"])


@pytest.mark.parametrize("name", golden_names("per_token_group_quant_int8"))
def test_per_token_group_quant_int8(name):
    meta, g = load_golden(name)
    q, s = modelnew("per_token_group_quant_int8", meta)(_as_dev(*g["x"]))
    _check(q, g["q"][0], "int8", {"max_abs_diff": 0})
    _check(s, g["scales"][0], "float32", TOL["FP32"])


@pytest.mark.parametrize("name", [n for n in golden_names("add_rmsnorm") if "fp8" not in n])
def test_add_rmsnorm(name):
    meta, g = load_golden(name)
    out = modelnew("add_rmsnorm", meta)(*(_as_dev(*g[k]) for k in ("x", "residual", "weight")))
    assert out.dtype == TORCH_DT[meta["dtype"]]
    _check(out, g["out"][0], "", TOL[meta["dtype"]])


@pytest.mark.parametrize("name", golden_names("int8_scaled_mm_azp"))
def test_int8_scaled_mm_azp(name):
    meta, g = load_golden(name)
    ins = [_as_dev(*g[k]) for k in ("a", "b", "a_scales", "b_scales", "azp_adj", "azp", "bias")]
    out = modelnew("int8_scaled_mm_azp", meta)(*ins)
    assert out.dtype == TORCH_DT[meta["output_dtype"]]
    _check(out, g["out"][0], "", TOL[meta["output_dtype"]])


@pytest.mark.parametrize("name", golden_names("paged_kv_cache_update"))
def test_paged_kv_cache_update(name):
    meta, g = load_golden(name)
    ins = [_as_dev(*g[k]) for k in ("to_cache", "kv_cache", "slot_mapping")]
    out = modelnew("paged_kv_cache_update", meta)(*ins)
    np.testing.assert_array_equal(host(out), g["out"][0].astype(np.float32))


@pytest.mark.parametrize("name", golden_names("paged_attention"))
def test_paged_attention_v1_v2(name):
    meta, g = load_golden(name)
    nb, bs, hkv, d = g["key_cache"][0].shape
    kc = _as_dev(*g["key_cache"]).view(nb, hkv, bs, d)
    vc = _as_dev(*g["value_cache"]).view(nb, hkv, bs, d)
    args = (_as_dev(*g["query"]), kc, vc, dev(g["seq_lens"][0]), dev(g["block_table"][0]))
    tol = TOL[meta["output_dtype"]]
    out = modelnew("paged_attention_v1", meta)(*args)
    _check(out, g["out_v1"][0], "", tol)
    o2, es, ml, tmp = modelnew("paged_attention_v2", meta)(*args)
    _check(o2, g["out_v2"][0], "", tol)
    _check(tmp, g["tmp_out"][0], "", tol)


@pytest.mark.parametrize("name", golden_names("batched_decode_attention"))
def test_batched_decode_attention(name):
    meta, g = load_golden(name)
    out = modelnew("batched_decode_attention", meta)(*(_as_dev(*g[k]) for k in ("q", "k_cache", "v_cache", "seq_lens")))
    _check(out, g["out"][0], "", TOL[meta["dtype"]])


@pytest.mark.parametrize("op,shape", [
    ("per_token_int8_quant", {"num_tokens": 2048, "hidden_dim": 4096, "dtype": "BF16"}),
    ("add_rmsnorm_fp8_quant", {"shape": [256, 8192], "eps": 1e-6, "dtype": "BF16"}),
    ("w8a8_scaled_mm", {"M": 256, "N": 4096, "K": 2048}),
    ("paged_fp8_decode", {"batch_size": 4, "num_q_heads": 32, "num_kv_heads": 8, "head_dim": 128, "block_size": 16,
                          "min_context": 100, "max_context": 700}),
])
def test_baseline_packages_model_vs_modelnew(op, shape):
    """The package's PyTorch Model (run on the GPU, as the harness does) against its ModelNew."""
    import importlib
    cat = {"per_token_int8_quant": "quantization", "add_rmsnorm_fp8_quant": "normalization",
           "w8a8_scaled_mm": "gemm", "paged_fp8_decode": "attention"}[op]
    mod = importlib.import_module(f"kernelverse_b200.operators.{cat}.{op}.{op}")
    torch.manual_seed(5)
    ins = [t.cuda() for t in mod.generate_inputs(shape)]
    ins2 = [t.clone() for t in ins]
    ref = mod.Model(shape)(*ins)
    got = modelnew(op, shape)(*ins2)
    refs = ref if isinstance(ref, tuple) else (ref,)
    gots = got if isinstance(got, tuple) else (got,)
    for r, o in zip(refs, gots):
        assert r.dtype == o.dtype and r.shape == o.shape
        if r.dtype == torch.float8_e4m3fn or (op == "add_rmsnorm_fp8_quant" and r.dtype == torch.uint8):
            from oracle import numerics
            d = np.abs(numerics.e4m3_ordinal(host(o)) - numerics.e4m3_ordinal(host(r)))
            assert d.max() <= 1
        elif r.dtype == torch.int8:
            assert (host(o).astype(np.int32) - host(r).astype(np.int32)).__abs__().max() <= 1
        else:
            np.testing.assert_allclose(host(o), host(r), rtol=1e-2, atol=1e-2)
    if op == "paged_fp8_decode":      # the fused write must leave the caches identical
        assert torch.equal(ins[1].view(torch.uint8), ins2[1].view(torch.uint8))
        assert torch.equal(ins[2].view(torch.uint8), ins2[2].view(torch.uint8))


@pytest.mark.parametrize("name", golden_names("static_scaled_int8_quant"))
def test_static_scaled_int8_quant(name):
    meta, g = load_golden(name)
    q = modelnew("static_scaled_int8_quant", meta)(_as_dev(*g["x"]), dev(g["scale"][0]), dev(g["azp"][0]))
    assert q.dtype == torch.int8
    _check(q, g["q"][0], "int8", {"max_abs_diff": 0})      # config.json allows 1; the kernel is exact


@pytest.mark.parametrize("name", golden_names("kv_cache_write"))
def test_kv_cache_write(name):
    meta, g = load_golden(name)
    ins = [_as_dev(*g[k]) for k in ("key_cache", "value_cache", "key", "value", "positions")]
    ko, vo = modelnew("kv_cache_write", meta)(*ins)
    np.testing.assert_array_equal(host(ko), g["key_out"][0].astype(np.float32))
    np.testing.assert_array_equal(host(vo), g["value_out"][0].astype(np.float32))


@pytest.mark.parametrize("name", golden_names("flash_decoding_attention"))
def test_flash_decoding_attention(name):
    meta, g = load_golden(name)
    outs = modelnew("flash_decoding_attention", meta)(*(_as_dev(*g[k]) for k in ("query", "key_cache", "value_cache")))
    tol = TOL[meta["dtype"]]
    for got, key in zip(outs, ("out", "exp_sums", "max_logits", "partial_out")):
        assert got.dtype == TORCH_DT[meta["dtype"]]
        ref = g[key][0].astype(np.float32)
        fin = np.isfinite(ref)
        assert np.array_equal(np.isfinite(host(got)), fin)
        np.testing.assert_allclose(host(got)[fin], ref[fin], rtol=tol["rtol"], atol=tol["atol"])


@pytest.mark.parametrize("name", golden_names("flash_attn_with_kvcache"))
def test_flash_attn_with_kvcache(name):
    meta, g = load_golden(name)
    out, lse = modelnew("flash_attn_with_kvcache", meta)(*(_as_dev(*g[k]) for k in ("q", "k_cache", "v_cache",
                                                                                       "cache_seqlens")))
    assert out.dtype == TORCH_DT[meta["dtype"]] and lse.dtype == torch.float32
    _check(out, g["out"][0], "", TOL[meta["dtype"]])
    _check(lse, g["softmax_lse"][0], "", TOL["FP32"] if meta["dtype"] == "FP32" else {"rtol": 2e-3, "atol": 2e-3})


@pytest.mark.parametrize("name", golden_names("batched_prefill_attention"))
def test_batched_prefill_attention(name):
    meta, g = load_golden(name)
    out = modelnew("batched_prefill_attention", meta)(*(_as_dev(*g[k]) for k in ("q", "k", "v", "qo_indptr",
                                                                                 "kv_indptr")))
    assert out.dtype == TORCH_DT[meta["dtype"]] and tuple(out.shape) == g["out"][0].shape
    _check(out, g["out"][0], "", TOL[meta["dtype"]])
