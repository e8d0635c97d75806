"""CPU checks of the drop-in boundary: ModelNew files, BASELINE operator packages, registry overlay."""
import importlib.util
import os
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from kernelverse_b200 import drop_in
from kernelverse_b200.registry_overlay import local_packages
from oracle import numerics, quant, rmsnorm

# The reference tree: KV_REFERENCE_ROOT, else the install made by baseline/install_ref.py.
_REF_ENV = os.environ.get("KV_REFERENCE_ROOT")
REF = Path(_REF_ENV) if _REF_ENV else Path(__file__).resolve().parents[1] / "baseline" / "_ref"
HAVE_REF = (REF / "operators" / "registry.py").exists()
# runner/generated_code_checker.py:101-112 (matched case-insensitively anywhere in the file)
BANNED = ("at::matmul", "at::softmax", "cublas", "cudnn", "cutlass", "hipblas", "miopen", "rocblas",
          "torch::matmul", "torch::softmax")


@pytest.mark.parametrize("op", drop_in.available())
def test_drop_in_files_define_modelnew_and_avoid_banned_words(op):
    code = drop_in.path(op).read_text()
    assert "class ModelNew" in code
    low = code.lower()
    assert not [w for w in BANNED if w in low]
    compile(code, str(drop_in.path(op)), "exec")


@pytest.mark.skipif(not HAVE_REF, reason="reference checker not available")
@pytest.mark.parametrize("op", drop_in.available())
def test_drop_in_files_pass_reference_static_checker(op):
    sys.path.insert(0, str(REF))
    try:
        from runner.generated_code_checker import check_generated_code
        report = check_generated_code(drop_in.path(op).read_text(), op_name=op)
    finally:
        sys.path.remove(str(REF))
    assert report["risk_level"] == "low", report


def test_every_package_has_a_drop_in():
    names = {op.name for _, op in local_packages()}
    assert names == {"per_token_int8_quant", "add_rmsnorm_fp8_quant", "w8a8_scaled_mm", "paged_fp8_decode"}
    assert names <= set(drop_in.available())


def _load(op_dir: Path):
    spec = importlib.util.spec_from_file_location(f"kvb_pkg_{op_dir.name}", op_dir / f"{op_dir.name}.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _pkg(name):
    for _, op in local_packages():
        if op.name == name:
            return _load(op)
    raise KeyError(name)


def test_package_per_token_int8_matches_oracle():
    m = _pkg("per_token_int8_quant")
    shape = {"num_tokens": 32, "hidden_dim": 512, "dtype": "BF16"}
    torch.manual_seed(0)
    (x,) = m.generate_inputs(shape)
    q, s = m.Model(shape)(x)
    rq, rs = quant.per_token_group_quant_int8(x.float().numpy(), 512, 1e-6)
    np.testing.assert_array_equal(q.numpy(), rq)
    np.testing.assert_array_equal(s.numpy(), rs[:, 0])


def test_package_add_rmsnorm_fp8_matches_oracle():
    m = _pkg("add_rmsnorm_fp8_quant")
    shape = {"shape": [8, 1024], "eps": 1e-6, "dtype": "BF16"}
    torch.manual_seed(1)
    x, r, w = m.generate_inputs(shape)
    ro, codes, scales = m.Model(shape)(x, r, w)
    er, ec, es, _ = rmsnorm.add_rmsnorm_quant(x.float().numpy(), r.float().numpy(), w.float().numpy(), 1e-6, "e4m3")
    np.testing.assert_array_equal(ro.float().numpy(), er)
    np.testing.assert_allclose(scales.numpy(), es, rtol=2e-6)
    d = np.abs(numerics.e4m3_ordinal(codes.view(torch.uint8).numpy()) - numerics.e4m3_ordinal(ec))
    assert d.max() <= 1


def test_package_w8a8_matches_oracle():
    from oracle import gemm
    m = _pkg("w8a8_scaled_mm")
    shape = {"M": 5, "N": 48, "K": 64}
    torch.manual_seed(2)
    a, b, sa, sb, bias = m.generate_inputs(shape)
    out = m.Model(shape)(a, b, sa, sb, bias)
    ref = gemm.w8a8_scaled_mm(a.numpy(), b.numpy(), sa.numpy(), sb.numpy(), bias.float().numpy(), "BF16")
    np.testing.assert_array_equal(out.float().numpy(), ref)


def test_package_paged_fp8_decode_matches_oracle():
    from oracle import attention, kv_cache
    m = _pkg("paged_fp8_decode")
    shape = {"batch_size": 3, "num_q_heads": 8, "num_kv_heads": 2, "head_dim": 64, "block_size": 16,
             "min_context": 1, "max_context": 70}
    torch.manual_seed(3)
    ins = m.generate_inputs(shape)
    q, kc, vc, ks, vs, lens, bt, kn, vn = ins
    kc0, vc0 = kc.view(torch.uint8).numpy().copy(), vc.view(torch.uint8).numpy().copy()
    out = m.Model(shape)(*ins)
    slots = kv_cache.decode_slots(lens.numpy(), bt.numpy(), 16)
    rk = kv_cache.paged_fp8_kv_write(kn.float().numpy(), kc0, slots, ks.numpy())
    rv = kv_cache.paged_fp8_kv_write(vn.float().numpy(), vc0, slots, vs.numpy())
    np.testing.assert_array_equal(kc.view(torch.uint8).numpy(), rk)
    ref = attention.paged_fp8_decode(q.float().numpy(), rk, rv, ks.numpy(), vs.numpy(), lens.numpy(), bt.numpy(),
                                     64 ** -0.5)
    np.testing.assert_allclose(out.float().numpy(), ref, rtol=1e-2, atol=1e-2)


@pytest.mark.skipif(not HAVE_REF, reason="reference registry not available")
def test_registry_overlay_discovers_packages():
    import subprocess
    code = ("import sys; sys.path.insert(0, %r);"
            "from operators.registry import get_operator_spec, list_operator_names;"
            "names = list_operator_names();"
            "assert 'w8a8_scaled_mm' in names and 'add_rmsnorm' in names, names;"
            "print(get_operator_spec('paged_fp8_decode')['category'])") % str(REF)
    root = Path(__file__).resolve().parents[1]
    env = dict(os.environ, PYTHONPATH=f"{root}/kernelverse_b200/overlay_site:{root}", PYTHONDONTWRITEBYTECODE="1")
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, env=env, timeout=120)
    assert r.returncode == 0, r.stderr
    assert r.stdout.strip() == "attention"
