"""CPU checks of the C ABI: libkvb.so loads, exports every symbol include/kvb.h declares,
the ctypes table mirrors the header, and argument validation fails cleanly without a GPU."""
import ctypes
import re
from pathlib import Path

import pytest

from kernelverse_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "kvb.h"


def header_functions():
    text = HEADER.read_text()
    return re.findall(r"KVB_API\s+[\w\s\*]+?\b(kvb_\w+)\s*\(", text)


def test_header_declares_functions():
    names = header_functions()
    assert "kvb_last_error" in names and len(names) >= 6
    assert len(names) == len(set(names))


def test_library_exports_every_header_symbol():
    lib = _lib.lib()
    for name in header_functions():
        assert hasattr(lib, name), name


def test_ctypes_table_matches_header():
    assert set(_lib.SIGNATURES) == set(header_functions())
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    for name, (_, argtypes) in _lib.SIGNATURES.items():
        m = re.search(rf"\b{name}\s*\(([^)]*)\)", text)
        params = [p for p in m.group(1).split(",") if p.strip() and p.strip() != "void"]
        assert len(params) == len(argtypes), name


def test_abi_version_and_error_string():
    lib = _lib.lib()
    assert lib.kvb_abi_version() >= 1
    assert isinstance(lib.kvb_last_error(), bytes)


def test_validation_errors_need_no_gpu():
    lib = _lib.lib()
    # hidden not divisible by group: rejected before any CUDA call
    rc = lib.kvb_per_token_group_quant_int8(None, _lib.BF16, 4, 100, 64, 1e-6, None, None, None)
    assert rc == 2 and b"multiple of group_size" in lib.kvb_last_error()
    rc = lib.kvb_dynamic_scaled_int8_quant(None, _lib.F32, -1, None, None, None, None, 0, None)
    assert rc == 1
    rc = lib.kvb_add_rmsnorm_quant(None, None, None, _lib.BF16, 2, 8, 1e-6, None, None, _lib.E4M3, None, None)
    assert rc == 1
    rc = lib.kvb_batched_prefill_attention(None, None, None, _lib.BF16, None, None, 1, 8, 8, 4, 3, 64, 0.125, None,
                                           None)
    assert rc == 2 and b"num_q_heads" in lib.kvb_last_error()
    rc = lib.kvb_batched_prefill_attention(None, None, None, _lib.BF16, None, None, 1, 8, 8, 4, 2, 136, 0.125, None,
                                           None)
    assert rc == 2 and b"head_dim" in lib.kvb_last_error()
    with pytest.raises(_lib.KvbError):
        _lib.call("kvb_per_token_group_quant_int8", None, _lib.F32, 1, 10, 3, 1e-6, None, None, None)


def test_ops_reject_cpu_tensors():
    import torch
    from kernelverse_b200 import ops
    with pytest.raises(ValueError, match="CUDA tensors only"):
        ops.per_token_group_quant_int8(torch.zeros(2, 8), 8, 1e-6)


def test_host_entry_argument_checks_need_no_gpu():
    """The host-buffer entry of the fused add+RMSNorm+quant takes host tensors of one shape; both
    checks run before any CUDA call."""
    import torch
    from kernelverse_b200 import ops
    x = torch.zeros(4, 64, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="same shape"):
        ops.add_rmsnorm_quant_host(x, torch.zeros(4, 32, dtype=torch.bfloat16), torch.ones(64), 1e-6)
    with pytest.raises(ValueError, match="same shape"):
        ops.add_rmsnorm_quant_host(x, torch.zeros(4, 64, dtype=torch.float16), torch.ones(64), 1e-6)
    with pytest.raises(ValueError, match="buffer slot"):
        ops.add_rmsnorm_quant_host(x, x.clone(), torch.ones(64), 1e-6, slots=0)


@pytest.mark.parametrize("rows,chunk,edge", [(0, 1, 256), (1, 1, 256), (7, 7, 256), (1024, 1024, 256),
                                             (1500, 1024, 256), (3000, 512, 256), (8192, 1024, 256),
                                             (8192, 1024, 1), (5000, 1000, 300)])
def test_host_entry_row_chunks(rows, chunk, edge):
    """The host-buffer entry's row chunks cover every row once, none larger than the buffer slots,
    short at both ends when the rows allow a ramp."""
    from kernelverse_b200.ops import _row_chunks
    sizes = _row_chunks(rows, chunk, edge)
    assert sum(sizes) == rows and all(0 < n <= chunk for n in sizes)
    if rows >= 4 * chunk and edge < chunk:
        assert sizes[0] == edge and sizes[-1] == edge and max(sizes) == chunk


@pytest.mark.parametrize("seqs,max_len,part", [(64, 8192, 512), (512, 8192, 512), (16, 4096, 128), (4, 4096, 64),
                                               (1, 100, 64), (8, 2048, 64), (0, 0, 64)])
def test_auto_partition_rule_needs_no_gpu(seqs, max_len, part):
    """partition_size 0: 512 tokens, halved down to 64 while sequences x partitions is below two
    per SM (148 SMs when no device answers, as here)."""
    from kernelverse_b200 import _lib
    assert _lib.lib().kvb_paged_attention_auto_partition(seqs, max_len) == part
