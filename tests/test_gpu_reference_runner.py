"""The reference's own correctness runner drives every drop-in ModelNew on the GPU, unchanged.

For each file in ``kernelverse_b200/drop_in/`` this calls KernelVerse's
``verify_generated_operator`` (runner/generated_correctness_runner.py:1813) for the operator's
``default`` single shape, language ``cuda``: the runner compiles the file through its ``cuda``
backend in a worker subprocess, runs seeded trials (seeds 1024 + 1000 * case + trial,
:1362-1363) with TF32 off, compares the outputs on the CPU under the category policies of
runner/correctness_policy.py:14-88 and the operator's tolerances, and profiles both models.
The reference is imported from ``baseline/_ref`` (installed by ``baseline/install_ref.py``);
``kernelverse_b200/overlay_site`` on ``PYTHONPATH`` lets its registry discover the four
BASELINE operator packages of this repository as well.
"""
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

from kernelverse_b200 import drop_in

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]
REF = ROOT / "baseline" / "_ref"

DRIVER = r"""
import json, sys
from runner.generated_correctness_runner import verify_generated_operator
op, path = sys.argv[1], sys.argv[2]
r = verify_generated_operator(op_name=op, language="cuda", shape_mode="single", shape_name="default",
                              shape_family="all", generated_path=path, device_id=0, trials=5, random_seed=None,
                              random_count=1, random_max_attempts=1, perf_trials=2)
c = r.get("correctness", {})
cases = r.get("cases") or [{}]
print("RESULT " + json.dumps({"compiled": r.get("compiled"), "success": c.get("success"),
                              "num_trials": c.get("num_trials"), "failed_trials": c.get("failed_trials"),
                              "error": c.get("error_message") or r.get("error_message"),
                              "case_keys": sorted(cases[0].keys())}))
"""


@pytest.mark.timeout(900)
@pytest.mark.parametrize("op", drop_in.available())
def test_reference_runner_accepts_drop_in(op):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    if not (REF / "runner" / "generated_correctness_runner.py").exists():
        pytest.skip("reference not installed in baseline/_ref (python baseline/install_ref.py)")
    env = dict(os.environ, PYTHONPATH=os.pathsep.join([str(ROOT / "kernelverse_b200" / "overlay_site"), str(ROOT),
                                                       str(REF)]),
               PYTHONDONTWRITEBYTECODE="1")
    r = subprocess.run([sys.executable, "-c", DRIVER, op, str(drop_in.path(op))], capture_output=True, text=True,
                       cwd=str(REF), env=env, timeout=840)
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("RESULT ")]
    assert r.returncode == 0 and lines, r.stdout[-3000:] + r.stderr[-3000:]
    res = json.loads(lines[-1][len("RESULT "):])
    assert res["compiled"] is True, res
    assert res["success"] is True and not res["failed_trials"], res
    assert res["num_trials"] == 5, res
