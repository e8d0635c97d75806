"""A bounded device-side wait that runs out: the kernel drains its copy, returns, and the host
sees status bit 0 and KVB_E_TIMEOUT; the context stays usable afterwards.

The wait is on an mbarrier on which nothing ever arrives (kvb_selftest_wait_timeout), with the
bound lowered to 2 ms for the test and restored afterwards.  No fault, trap or endless loop.
"""
import time

import pytest
import torch

from gpu_util import require_gpu

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_drains_and_reports_timeout():
    require_gpu()
    from kernelverse_b200 import _lib, ops
    lib = _lib.lib()
    lib.kvb_device_status(1)
    src = torch.tensor([0x5EED, 1, 2, 3], dtype=torch.int32, device="cuda")
    out = torch.zeros(3, dtype=torch.int32, device="cuda")
    _lib.call("kvb_set_wait_limit_ns", 2_000_000)
    try:
        t0 = time.perf_counter()
        _lib.call("kvb_selftest_wait_timeout", src.data_ptr(), out.data_ptr(), torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
    finally:
        _lib.call("kvb_set_wait_limit_ns", 0)
    assert out.tolist() == [0x5EED, 1, 1]            # copied word, gave up, drained
    assert dt < 1.0                                   # the lowered bound, not the 2 s default
    assert lib.kvb_device_status(0) & 1
    assert lib.kvb_check_device(1) == 6               # KVB_E_TIMEOUT, and the words are cleared
    assert b"bounded device-side wait" in lib.kvb_last_error()
    assert lib.kvb_device_status(0) == 0
    # the context is still usable: a real kernel runs and the status stays clean
    x = torch.randn(8, 256, device="cuda").to(torch.bfloat16)
    q, s = ops.per_token_group_quant_int8(x, 256, 1e-6)
    torch.cuda.synchronize()
    assert q.shape == (8, 256) and torch.isfinite(s).all()
    _lib.check_device()


def test_wait_selftest_rejects_a_misaligned_source():
    require_gpu()
    from kernelverse_b200 import _lib
    src = torch.arange(8, dtype=torch.int32, device="cuda")
    out = torch.zeros(3, dtype=torch.int32, device="cuda")
    with pytest.raises(_lib.KvbError):
        _lib.call("kvb_selftest_wait_timeout", src.data_ptr() + 4, out.data_ptr(), 0)
    assert _lib.lib().kvb_device_status(1) == 0
