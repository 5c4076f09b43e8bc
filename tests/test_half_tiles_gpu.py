"""GPU: the M = 64 tile variant of the grouped GEMMs (MOE_HALF_TILES=1): an
m-block whose rows 64..127 are all padding runs half-height MMAs (bf16, f16
and int8; block-scaled MMAs exist with M = 128 only, so the UE8M0 kernel
ignores the switch, which a UE8M0 case checks). The layer must match the
fp32 oracle within the bf16 tolerance and agree with the default M = 128
path (run in a child process without the switch).
"""
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

TOL = dict(rtol=2e-2, atol=2e-2)
ROOT = Path(__file__).resolve().parent.parent

CASES = [
    # T, H, I, E, k, quant: every block a tail (few rows per expert), mixed
    # full and half blocks, int8, and a K-split down GEMM (decode-sized)
    (50, 256, 256, 16, 4, "none"),
    (1024, 512, 256, 64, 8, "none"),
    (300, 256, 256, 16, 4, "int8"),
    (20, 512, 512, 8, 2, "none"),
    (200, 256, 256, 16, 4, "fp8-ue8m0"),  # the block-scaled kernel's M = 64 tiles
]


def run_case(T, H, I, E, k, quant):
    from kernelswift_b200 import fused_moe as fm
    from oracle import moe_oracle as orc

    dev = torch.device("cuda", 0)
    g = torch.Generator().manual_seed(T * 7 + E)
    hidden = torch.randn(T, H, generator=g).to(torch.bfloat16)
    w, ids = orc.route(torch.randn(T, E, generator=g) + torch.linspace(0, 1, E), k)
    w1 = torch.randn(E, 2 * I, H, generator=g) / H ** 0.5
    w2 = torch.randn(E, H, I, generator=g) / I ** 0.5
    out = fm.fused_experts(hidden.to(dev), w1.to(dev), w2.to(dev), w.to(dev), ids.to(dev),
                           use_int8_w8a8=quant == "int8", use_fp8_w8a8=quant == "fp8-ue8m0",
                           scale_format="ue8m0")
    torch.cuda.synchronize()
    return out.cpu(), hidden, w1, w2, w, ids


def child(case, path, half):
    code = (f"import sys, torch\nsys.path.insert(0, {str(ROOT)!r})\n"
            f"sys.path.insert(0, {str(ROOT / 'tests')!r})\n"
            f"from test_half_tiles_gpu import run_case\n"
            f"torch.save(run_case(*{case!r})[0], {str(path)!r})\n")
    env = dict(os.environ, MOE_HALF_TILES="1" if half else "0")
    res = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True,
                         timeout=600)
    assert res.returncode == 0, res.stderr[-2000:]
    return torch.load(path)


@pytest.mark.parametrize("case", CASES, ids=[f"T{c[0]}_E{c[3]}_k{c[4]}_{c[5]}" for c in CASES])
def test_half_tiles_match_oracle_and_default(cuda_device, tmp_path, case):
    from oracle import moe_oracle as orc

    half = child(case, tmp_path / "half.pt", True)
    full = child(case, tmp_path / "full.pt", False)
    _, hidden, w1, w2, w, ids = run_case(*case)
    if case[5] in ("int8", "fp8-ue8m0"):
        f = orc.fused_experts_int8 if case[5] == "int8" else orc.fused_experts_fp8_ue8m0
        ref = f(hidden, w1, w2, w, ids)
        assert orc.rel_l2(half, ref) <= 5e-2
    else:
        ref = orc.fused_experts(hidden.float(), w1, w2, w, ids)
        torch.testing.assert_close(half.float(), ref, **TOL)
    torch.testing.assert_close(half.float(), full.float(), **TOL)
