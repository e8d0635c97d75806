import json
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) and the built libkvb.so")


def load_golden(name: str):
    """Load one fixture: returns (meta dict, {name: (array, torch-dtype-name)}).

    bf16 arrays come back as float32 values, float8_e4m3fn arrays as uint8 codes.
    """
    from oracle.numerics import bf16_bits_to_f32

    z = np.load(GOLDEN / f"{name}.npz")
    meta = json.loads(str(z["meta"]))
    out = {}
    for k in z.files:
        if k.endswith("__dtype") or k == "meta":
            continue
        dt = str(z[k + "__dtype"]) if (k + "__dtype") in z.files else None
        a = z[k]
        if dt == "bfloat16":
            a = bf16_bits_to_f32(a)
        out[k] = (a, dt)
    return meta, out


def golden_names(prefix: str):
    """Fixtures named ``<prefix>_<number>`` (so ``w8a8`` does not also pick up ``w8a8_act_0``)."""
    return sorted(p.stem for p in GOLDEN.glob(f"{prefix}_*.npz") if p.stem[len(prefix) + 1:].isdigit())


@pytest.fixture
def golden():
    return load_golden


@pytest.fixture(autouse=True)
def _device_status_clean(request):
    """GPU tests: no bounded device-side wait may have given up during the test."""
    yield
    if request.node.get_closest_marker("gpu") is None:
        return
    import torch
    if not torch.cuda.is_available():
        return
    from kernelverse_b200 import _lib
    status = _lib.lib().kvb_device_status(1)
    assert status == 0, f"kvb_device_status = {status:#x} after {request.node.name}"
