"""GPU: the token-major gather writes the same operand rows as the row-major one.

moe_fused_experts gathers (and for fp8 quantises) the routed rows through
the align's slot map, reading each token once and storing it into its
top_k operand rows. MOE_NO_TOKEN_GATHER=1 restores the row-major gather,
which reads the source once per routed row. Every element goes through the
same arithmetic in both, so the layer outputs must be equal bit for bit.
Both variants run in child processes (the switch is read once per
process) over bf16, f16, fp32 (tf32 operands), fp8 with fp32 block scales
and fp8 with UE8M0 scales, with dropped slots (ids -1 and E), int64 ids,
H that are not multiples of the 1024-column chunk (an odd number of
128-column groups in fp8, H = 1152), and a device-side token count that
leaves the tail of the batch out.
"""
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent

# name: (T, H, I, E, k, quant, activation dtype, scale format, options)
PROBLEMS = {
    "bf16_k8": (300, 2048, 768, 16, 8, "none", torch.bfloat16, None, {}),
    "bf16_k2_dropped": (257, 1536, 512, 8, 2, "none", torch.bfloat16, None, {"drop": True}),
    "f16_k4": (129, 1024, 512, 8, 4, "none", torch.float16, None, {"i64": True}),
    "tf32_k2": (200, 1024, 512, 8, 2, "none", torch.float32, None, {}),
    "fp8_k8": (300, 1792, 512, 16, 8, "fp8", torch.bfloat16, "fp32", {}),
    "fp8_odd_groups": (100, 1152, 512, 8, 2, "fp8", torch.bfloat16, "fp32", {}),
    "ue8m0_k8": (500, 7168, 512, 32, 8, "fp8-ue8m0", torch.bfloat16, "ue8m0", {"drop": True}),
    "ue8m0_count": (400, 2048, 512, 16, 8, "fp8-ue8m0", torch.bfloat16, "ue8m0",
                    {"count": 301}),
}


def compute(name, device):
    from kernelswift_b200 import fused_moe as fm

    T, H, I, E, k, quant, dtype, fmt, opt = PROBLEMS[name]
    g = torch.Generator(device=device).manual_seed(sum(map(ord, name)))
    hidden = torch.randn(T, H, generator=g, device=device).to(dtype)
    logits = torch.randn(T, E, generator=g, device=device)
    w1 = torch.randn(E, 2 * I, H, generator=g, device=device) / H ** 0.5
    w2 = torch.randn(E, H, I, generator=g, device=device) / I ** 0.5
    prep = fm.prepare_weights(w1, w2, quant, fm.compute_dtype_for(dtype, quant))
    with torch.no_grad():
        tw, ti = fm.fused_topk(hidden, logits, k, weights_dtype=dtype)
        if opt.get("drop"):
            ti[1, 0] = -1
            ti[T // 2, k - 1] = E
        if opt.get("i64"):
            ti = ti.long()
        count = None
        if "count" in opt:
            count = torch.tensor([opt["count"]], dtype=torch.int32, device=device)
        out = torch.zeros(T, H, dtype=dtype, device=device)
        kw = {"use_fp8_w8a8": quant.startswith("fp8")}
        if fmt is not None:
            kw["scale_format"] = fmt
        fm.fused_experts(hidden, prep, None, tw, ti, out=out, num_tokens_dev=count, **kw)
    torch.cuda.synchronize(device)
    return out.cpu()


CHILD = """
import sys, torch
sys.path.insert(0, {root!r}); sys.path.insert(0, {tests!r})
from test_token_gather_gpu import PROBLEMS, compute
dev = torch.device("cuda", 0)
torch.save({{n: compute(n, dev) for n in PROBLEMS}}, {out!r})
"""


def run_child(tmp, extra_env):
    out = tmp / ("r%d.pt" % len(extra_env))
    env = dict(os.environ, **extra_env)
    code = CHILD.format(root=str(ROOT), tests=str(ROOT / "tests"), out=str(out))
    res = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True,
                         text=True, timeout=900)
    assert res.returncode == 0, res.stderr[-2000:]
    return torch.load(out)


@pytest.fixture(scope="module")
def both(cuda_device, tmp_path_factory):
    tmp = tmp_path_factory.mktemp("token_gather")
    return run_child(tmp, {}), run_child(tmp, {"MOE_NO_TOKEN_GATHER": "1"})


@pytest.mark.parametrize("name", sorted(PROBLEMS))
def test_token_gather_matches_row_gather(cuda_device, both, name):
    tok, row = both[0][name], both[1][name]
    assert torch.isfinite(tok.float()).all()
    assert tok.abs().sum() > 0
    assert torch.equal(tok, row), name
    opt = PROBLEMS[name][-1]
    if "count" in opt:
        assert not tok[opt["count"]:].any()  # rows past the count untouched (zero)
