"""GPU: the device-timed v0/v1 runner on a B200, the way auto_bench compares
a candidate with base.py (auto_bench.py:637-695): the drop-in v1 module
(kernelswift_b200/ks_fused_moe.py) against the oracle's restatement of
base.py's Model at base.py's default problem (tests/golden/oracle_v0_module.py),
through the runner's command line, which prints one JSON line."""
import json
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent


def test_runner_prints_device_timed_match(cuda_device):
    cmd = [sys.executable, "-m", "kernelswift_b200.ab_runner",
           "--v0_file", str(ROOT / "tests" / "golden" / "oracle_v0_module.py"),
           "--v1_file", str(ROOT / "kernelswift_b200" / "ks_fused_moe.py"),
           "--warmup", "5", "--repeat", "20"]
    res = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=600,
                         env={**__import__("os").environ, "PYTHONPATH": str(ROOT)})
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [ln for ln in res.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, res.stdout
    r = json.loads(lines[0])
    print(lines[0])
    assert r["device"].startswith("cuda") and r["timing"] == "CUDA events, median"
    # auto_bench's criterion: allclose(atol=rtol=1e-2) on v0's inputs
    assert r["match"], r["differences"]
    assert r["v0_ms"] > 0 and r["v1_ms"] > 0
