"""GPU: tail halves of the rows GEMM do not change results.

With 256-wide unsplit tiles, when the tiles leave the last wave of CTAs at
most half full, the grouped down GEMM runs those last tiles as two 128-column
halves each (the last wave then takes about half a tile-time). Every output
element keeps its K order, so the layer's output is the same bit for bit as
with full-width tiles only. Both variants run in child processes with
MOE_BLOCK_N=256 (so that small problems also take 256-wide tiles), one of
them with MOE_NO_TAIL_HALVES=1, and their outputs are compared. The small
problems have 64 tiles (16 m-blocks x 4 column tiles), so the halves always
engage; at the Mixtral layer (about 67 m-blocks x 16) they engage unless the
routing puts the remainder above 74.
"""
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent

# name: (T, H, I, E, k, quant, activation dtype)
PROBLEMS = {
    "mixtral_T4096": (4096, 4096, 14336, 8, 2, "none", torch.bfloat16),
    "bf16_T600": (600, 1024, 512, 8, 2, "none", torch.bfloat16),
    "f16_T600": (600, 1024, 512, 8, 2, "none", torch.float16),
    "tf32_T600": (600, 1024, 512, 8, 2, "none", torch.float32),
    "int8_T600": (600, 1024, 512, 8, 2, "int8", torch.bfloat16),
}
ALWAYS_ENGAGED = {"bf16_T600", "f16_T600", "tf32_T600", "int8_T600"}


def compute(name, device):
    """(output, down-GEMM plan, tile remainder over the SMs) of one problem."""
    from kernelswift_b200 import fused_moe as fm

    T, H, I, E, k, quant, dtype = PROBLEMS[name]
    g = torch.Generator(device=device).manual_seed(sum(map(ord, name)))
    hidden = torch.randn(T, H, generator=g, device=device).to(dtype)
    logits = torch.randn(T, E, generator=g, device=device)
    w1 = torch.randn(E, 2 * I, H, generator=g, device=device) / H ** 0.5
    w2 = torch.randn(E, H, I, generator=g, device=device) / I ** 0.5
    prep = fm.prepare_weights(w1, w2, quant, fm.compute_dtype_for(dtype, quant))
    with torch.no_grad():
        tw, ti = fm.fused_topk(hidden, logits, k, weights_dtype=dtype)
        out = fm.fused_experts(hidden, prep, None, tw, ti, use_int8_w8a8=quant == "int8")
    torch.cuda.synchronize(device)
    plan = fm.fused_experts_plan(T, H, I, E, k, quant, dtype)
    counts = torch.bincount(ti.reshape(-1).long().cpu(), minlength=E)
    m_blocks = int(((counts + 127) // 128).sum())
    rem = (m_blocks * (H // 256)) % plan["sms"]
    return {"out": out.cpu(), "plan": plan, "rem": rem}


CHILD = """
import sys, torch
sys.path.insert(0, {root!r}); sys.path.insert(0, {tests!r})
from test_tail_halves_gpu import PROBLEMS, compute
dev = torch.device("cuda", 0)
torch.save({{n: compute(n, dev) for n in PROBLEMS}}, {out!r})
"""


def run_child(tmp, extra_env):
    out = tmp / ("r%d.pt" % len(extra_env))
    env = dict(os.environ, MOE_BLOCK_N="256", **extra_env)
    code = CHILD.format(root=str(ROOT), tests=str(ROOT / "tests"), out=str(out))
    res = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True,
                         text=True, timeout=900)
    assert res.returncode == 0, res.stderr[-2000:]
    return torch.load(out)


@pytest.fixture(scope="module")
def both(cuda_device, tmp_path_factory):
    tmp = tmp_path_factory.mktemp("halves")
    return run_child(tmp, {}), run_child(tmp, {"MOE_NO_TAIL_HALVES": "1"})


@pytest.mark.parametrize("name", sorted(PROBLEMS))
def test_tail_halves_match_full_width_tiles(cuda_device, both, name):
    halves, full = both[0][name], both[1][name]
    assert halves["plan"]["down_block_n"] == 256 and halves["plan"]["down_splits"] == 1
    if name in ALWAYS_ENGAGED:
        assert 0 < halves["rem"] and 2 * halves["rem"] <= halves["plan"]["sms"], halves["rem"]
    assert torch.isfinite(halves["out"].float()).all()
    assert torch.equal(halves["out"], full["out"]), name
