"""GPU: the gate-up GEMM that gathers its own A rows (MOE_GATHER_TMA=1):
each A tile is loaded from the token matrix by TMA tile::gather4 (token
sorted_ids[m] / top_k, four rows per instruction) instead of from the copy a
gather pass writes. The operand values and the MMA order are the same, so
the layer must equal the default path bit for bit (child process without
the switch) and match the fp32 oracle within the bf16 tolerance.

The variant has not yet been run on a B200, so these tests only run with
MOE_TEST_GATHER_TMA=1 until it has passed them there once.
"""
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(os.environ.get("MOE_TEST_GATHER_TMA") != "1",
                       reason="gathered gate-up A rows not yet run on a B200; "
                              "set MOE_TEST_GATHER_TMA=1 to run it"),
]

TOL = dict(rtol=2e-2, atol=2e-2)
ROOT = Path(__file__).resolve().parent.parent

CASES = [
    # T, H, I, E, k, dtype: tail blocks only, many experts, 256-wide tiles,
    # f16, an uneven token count (rows 4l..4l+3 cross tokens), Qwen3-shaped
    (50, 256, 256, 16, 4, "bf16"),
    (1024, 512, 256, 64, 8, "bf16"),
    (700, 1024, 512, 8, 2, "bf16"),
    (200, 256, 256, 8, 2, "f16"),
    (129, 384, 128, 8, 2, "bf16"),
    (4096, 2048, 768, 128, 8, "bf16"),
]
DTYPES = {"bf16": torch.bfloat16, "f16": torch.float16}


def problem(T, H, I, E, k, dtype):
    from oracle import moe_oracle as orc

    g = torch.Generator().manual_seed(T * 13 + E)
    w, ids = orc.route(torch.randn(T, E, generator=g) + torch.linspace(0, 1, E), k)
    hidden = torch.randn(T, H, generator=g).to(DTYPES[dtype])
    w1 = torch.randn(E, 2 * I, H, generator=g) / H ** 0.5
    w2 = torch.randn(E, H, I, generator=g) / I ** 0.5
    return hidden, w1, w2, w, ids


def run_case(T, H, I, E, k, dtype):
    from kernelswift_b200 import fused_moe as fm

    dev = torch.device("cuda", 0)
    hidden, w1, w2, w, ids = problem(T, H, I, E, k, dtype)
    out = fm.fused_experts(hidden.to(dev), w1.to(dev), w2.to(dev), w.to(dev), ids.to(dev))
    torch.cuda.synchronize()
    return out.cpu()


def child(case, path, env_extra):
    code = (f"import sys, torch\nsys.path.insert(0, {str(ROOT)!r})\n"
            f"sys.path.insert(0, {str(ROOT / 'tests')!r})\n"
            f"from test_gather_tma_gpu import run_case\n"
            f"torch.save(run_case(*{case!r}), {str(path)!r})\n")
    env = dict(os.environ, **env_extra)
    res = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True,
                         timeout=600)
    assert res.returncode == 0, res.stderr[-2000:]
    return torch.load(path)


@pytest.mark.parametrize("case", CASES, ids=[f"T{c[0]}_H{c[1]}_E{c[3]}_k{c[4]}_{c[5]}"
                                             for c in CASES])
def test_gathered_rows_match_default_and_oracle(cuda_device, tmp_path, case):
    from kernelswift_b200 import fused_moe as fm
    from oracle import moe_oracle as orc

    T, H, I, E, k, dtype = case
    assert fm.fused_experts_plan(T, H, I, E, k, dtype=DTYPES[dtype])["gate_up_splits"] == 1
    gathered = child(case, tmp_path / "g.pt", {"MOE_GATHER_TMA": "1"})
    plain = child(case, tmp_path / "p.pt", {"MOE_GATHER_TMA": "0"})
    assert torch.equal(gathered, plain)
    hidden, w1, w2, w, ids = problem(*case)
    ref = orc.fused_experts(hidden.float(), w1, w2, w, ids)
    torch.testing.assert_close(gathered.float(), ref, **TOL)


def test_gathered_rows_with_half_tiles(cuda_device, tmp_path):
    case = CASES[1]
    both = child(case, tmp_path / "b.pt", {"MOE_GATHER_TMA": "1", "MOE_HALF_TILES": "1"})
    plain = child(case, tmp_path / "p.pt", {"MOE_GATHER_TMA": "0", "MOE_HALF_TILES": "1"})
    assert torch.equal(both, plain)
