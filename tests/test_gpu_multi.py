"""Multi-GPU path on real GPUs (skipped on boxes with fewer than two): the fused
column-sharded TP GEMM + all-gather equals the single-GPU GEMM bit for bit."""
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.timeout(600)
def test_tp_gemm_allgather_two_gpus():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={_port()}", str(ROOT / "tests" / "mgpu" / "tp_gemm_check.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, cwd=ROOT, timeout=400)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "TP_OK" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]


@pytest.mark.timeout(900)
def test_tp_gemm_allgather_all_gpus():
    """The same check with one rank per GPU of the box (4 or 8 on a multi-GPU box)."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < 4:
        pytest.skip("needs four or more GPUs")
    n = torch.cuda.device_count()
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={n}", "--master-addr=127.0.0.1", f"--master-port={_port()}",
           str(ROOT / "tests" / "mgpu" / "tp_gemm_check.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, cwd=ROOT, timeout=700)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert r.stdout.count("TP_OK") >= 1, r.stdout[-3000:] + r.stderr[-3000:]
