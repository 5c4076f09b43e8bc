"""GPU: programmatic dependent launch does not change results.

Every kernel of the forward may start before its predecessor in the stream
has finished (griddepcontrol), and the grouped GEMMs read the align metadata
and request their first weight tiles before waiting on the kernel that
writes their A operand. The same problems are computed in a child process
with MOE_NO_PDL=1 (plain stream ordering) and compared bit for bit with this
process's results, eagerly and replayed from a CUDA graph, for decode-sized
(split-K) and larger (single-pass) plans, bf16 and fp8.
"""
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

from kernelswift_b200 import fused_moe as fm

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent

# name: (T, H, I, E, k, quant)
PROBLEMS = {
    "decode_bf16": (3, 256, 128, 8, 2, "none"),
    "mid_bf16": (300, 512, 256, 16, 4, "none"),
    "decode_fp8": (40, 512, 256, 8, 2, "fp8"),
}


def compute(name, device):
    """Eager and graph-replayed outputs of one problem (seeded on the CPU)."""
    T, H, I, E, k, quant = PROBLEMS[name]
    g = torch.Generator().manual_seed(sum(map(ord, name)))
    hidden = torch.randn(T, H, generator=g).to(torch.bfloat16).to(device)
    logits = torch.randn(T, E, generator=g).to(device)
    w1 = (torch.randn(E, 2 * I, H, generator=g) / H ** 0.5).to(torch.bfloat16).to(device)
    w2 = (torch.randn(E, H, I, generator=g) / I ** 0.5).to(torch.bfloat16).to(device)
    prep = fm.prepare_weights(w1, w2, quant, torch.bfloat16)

    def fwd(hd, ld):
        tw, ti = fm.fused_topk(hd, ld, k, weights_dtype=hd.dtype)
        return fm.fused_experts(hd, prep, None, tw, ti, use_fp8_w8a8=quant == "fp8")

    with torch.no_grad():
        eager = fwd(hidden, logits).clone()
        cap = fm.CapturedMoE(fwd, T, H, E, dtype=torch.bfloat16, device=device)
        graph = cap(hidden, logits).clone()
    torch.cuda.synchronize(device)
    return {"eager": eager.cpu(), "graph": graph.cpu()}


CHILD = """
import sys, torch
sys.path.insert(0, {root!r}); sys.path.insert(0, {tests!r})
from test_pdl_gpu import PROBLEMS, compute
dev = torch.device("cuda", 0)
torch.save({{n: compute(n, dev) for n in PROBLEMS}}, {out!r})
"""


@pytest.fixture(scope="module")
def plain_results(cuda_device, tmp_path_factory):
    out = tmp_path_factory.mktemp("pdl") / "plain.pt"
    env = dict(os.environ, MOE_NO_PDL="1")
    code = CHILD.format(root=str(ROOT), tests=str(ROOT / "tests"), out=str(out))
    res = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True,
                         text=True, timeout=600)
    assert res.returncode == 0, res.stderr[-2000:]
    return torch.load(out)


@pytest.mark.parametrize("name", sorted(PROBLEMS))
def test_pdl_matches_plain_launches(cuda_device, plain_results, name):
    ours = compute(name, cuda_device)
    for mode in ("eager", "graph"):
        assert torch.isfinite(ours[mode].float()).all()
        assert torch.equal(ours[mode], plain_results[name][mode]), (name, mode)
    assert torch.equal(ours["eager"], ours["graph"]), name
