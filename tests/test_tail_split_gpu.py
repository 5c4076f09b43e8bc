"""GPU: the tail split of the down GEMM (MOE_TAIL_SPLIT=1): the tiles of the
last partial wave are split along K over the otherwise idle SMs, and the part
that completes a tile last adds the parts in part order. The layer must match
the fp32 oracle within the bf16 tolerance (int8: 5e-2 relative L2 against
the dequantised oracle), agree with the default path (child process without
the switch), and repeat bit for bit.
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
SMS = 148

CASES = [
    # T, H, I, E, k, quant: down tile width / tiles / tail tiles / parts with
    # this routing are checked by tail_shape() below
    (900, 2048, 1024, 16, 2, "none"),    # 256-wide, 168 tiles, 20 in the tail, 7 parts
    (1200, 1024, 1024, 8, 4, "none"),    # 128-wide, 328 tiles, 32 in the tail, 4 parts
    (600, 1024, 512, 16, 2, "none"),     # one partial wave: every tile split in 2
    (1200, 2048, 512, 8, 2, "int8"),     # kind::i8: parts added as int32
]


def problem(T, H, I, E, k):
    from oracle import moe_oracle as orc

    g = torch.Generator().manual_seed(T * 7 + E)
    w, ids = orc.route(torch.randn(T, E, generator=g) + torch.linspace(0, 1, E), k)
    hidden = torch.randn(T, H, generator=g).to(torch.bfloat16)
    w1 = torch.randn(E, 2 * I, H, generator=g) / H ** 0.5
    w2 = torch.randn(E, H, I, generator=g) / I ** 0.5
    return hidden, w1, w2, w, ids


def tail_shape(T, H, I, E, k, quant):
    """(tiles, tail tiles, parts) of the down GEMM for the case's routing."""
    from kernelswift_b200 import fused_moe as fm

    _, _, _, _, ids = problem(T, H, I, E, k)
    cnt = torch.bincount(ids.reshape(-1), minlength=E)
    mb = int(((cnt + 127) // 128).sum())
    plan = fm.fused_experts_plan(T, H, I, E, k, quant)
    assert plan["down_splits"] == 1
    tiles = mb * (H // plan["down_block_n"])
    tail = tiles % SMS
    k_blocks = -(-I * (2 if quant == "none" else 1) // 128)
    return tiles, tail, min(SMS // tail, k_blocks) if tail else 0


def run_case(T, H, I, E, k, quant):
    from kernelswift_b200 import fused_moe as fm

    dev = torch.device("cuda", 0)
    hidden, w1, w2, w, ids = problem(T, H, I, E, k)
    args = (hidden.to(dev), w1.to(dev), w2.to(dev), w.to(dev), ids.to(dev))
    a = fm.fused_experts(*args, use_int8_w8a8=quant == "int8")
    b = fm.fused_experts(*args, use_int8_w8a8=quant == "int8")
    torch.cuda.synchronize()
    assert torch.equal(a, b), "not deterministic"
    return a.cpu()


def child(case, path, env_extra):
    code = (f"import sys, torch\nsys.path.insert(0, {str(ROOT)!r})\n"
            f"sys.path.insert(0, {str(ROOT / 'tests')!r})\n"
            f"from test_tail_split_gpu import run_case\n"
            f"torch.save(run_case(*{case!r}), {str(path)!r})\n")
    env = dict(os.environ, **env_extra)
    res = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True,
                         timeout=600)
    assert res.returncode == 0, res.stderr[-2000:]
    return torch.load(path)


@pytest.mark.parametrize("case", CASES, ids=[f"T{c[0]}_H{c[1]}_E{c[3]}_k{c[4]}_{c[5]}"
                                             for c in CASES])
def test_tail_split_matches_oracle_and_default(cuda_device, tmp_path, case):
    from oracle import moe_oracle as orc

    tiles, tail, parts = tail_shape(*case)
    assert tail > 0 and parts >= 2, (tiles, tail, parts)  # the case exercises the split
    split = child(case, tmp_path / "tail.pt", {"MOE_TAIL_SPLIT": "1"})
    plain = child(case, tmp_path / "plain.pt", {"MOE_TAIL_SPLIT": "0"})
    hidden, w1, w2, w, ids = problem(*case[:5])
    if case[5] == "int8":
        ref = orc.fused_experts_int8(hidden, w1, w2, w, ids)
        assert orc.rel_l2(split, ref) <= 5e-2
        assert torch.equal(split, plain)  # int32 parts add exactly
    else:
        ref = orc.fused_experts(hidden.float(), w1, w2, w, ids)
        torch.testing.assert_close(split.float(), ref, **TOL)
        torch.testing.assert_close(split.float(), plain.float(), **TOL)


def test_tail_split_with_half_tiles(cuda_device, tmp_path):
    case = CASES[0]
    both = child(case, tmp_path / "both.pt", {"MOE_TAIL_SPLIT": "1", "MOE_HALF_TILES": "1"})
    plain = child(case, tmp_path / "plain.pt", {"MOE_TAIL_SPLIT": "0", "MOE_HALF_TILES": "0"})
    torch.testing.assert_close(both.float(), plain.float(), **TOL)
