"""Helpers shared by the GPU parity tests."""
import numpy as np
import pytest
import torch

TORCH_DT = {"FP32": torch.float32, "FP16": torch.float16, "BF16": torch.bfloat16,
            "float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}


def require_gpu():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    major, minor = torch.cuda.get_device_capability()
    assert major == 10, f"kernels are built for sm_100a, device is sm_{major}{minor}"


def dev(a, dtype=None):
    """numpy -> CUDA tensor; float arrays are cast to ``dtype`` (exact for representable values)."""
    a = np.ascontiguousarray(a)
    t = torch.from_numpy(a)
    if dtype is not None:
        t = t.to(dtype)
    return t.cuda()


def host(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu()
    if t.dtype == torch.float8_e4m3fn:
        return t.view(torch.uint8).numpy()
    if t.dtype in (torch.bfloat16, torch.float16):
        return t.float().numpy()
    return t.numpy()


def seeded(seed: int) -> np.random.Generator:
    return np.random.default_rng(seed)


def bf16_normal(rng, shape, std=1.0, mean=0.0):
    """float32 array of bf16-representable N(mean, std) values."""
    from oracle.numerics import round_bf16
    return round_bf16((rng.standard_normal(shape) * std + mean).astype(np.float32))
