"""GPU: moe_align_block_size is bit-exact with the oracle's counting sort."""
import numpy as np
import pytest
import torch

from cases import CASES
from kernelswift_b200 import fused_moe as fm
from oracle import moe_oracle as orc

pytestmark = pytest.mark.gpu

GOLDEN = __import__("pathlib").Path(__file__).resolve().parent / "golden"


def run_and_compare(ids: torch.Tensor, E: int, bm: int):
    s, e, n = fm.moe_align_block_size(ids, bm, E)
    torch.cuda.synchronize()
    rs, re_, rn = orc.moe_align(ids.cpu(), E, bm)
    assert int(n.item()) == rn
    assert np.array_equal(s.cpu().numpy(), rs)
    assert np.array_equal(e.cpu().numpy(), re_)


def gen_ids(kind, T, k, E, seed, dtype=torch.int64):
    g = torch.Generator().manual_seed(seed)
    if kind == "topk":
        logits = torch.randn(T, E, generator=g)
        ids = torch.topk(logits, min(k, E), dim=-1).indices
    elif kind == "skewed":
        logits = torch.randn(T, E, generator=g) + torch.randn(E, generator=g) * 2.0
        ids = torch.topk(logits, min(k, E), dim=-1).indices
    elif kind == "one_expert":
        ids = torch.full((T, k), E - 1, dtype=torch.int64)
    elif kind == "uniform":
        ids = torch.randint(0, E, (T, k), generator=g)
    elif kind == "with_invalid":
        ids = torch.randint(-1, E + 2, (T, k), generator=g)
    else:
        raise ValueError(kind)
    return ids.to(dtype)


SHAPES = [
    # (kind, T, k, E, block_m)
    ("topk", 1, 2, 8, 128),
    ("topk", 1, 8, 256, 128),
    ("topk", 3, 8, 128, 64),
    ("topk", 17, 2, 8, 16),
    ("topk", 64, 8, 256, 128),      # E > T*k
    ("skewed", 1024, 8, 128, 128),
    ("one_expert", 300, 2, 8, 128),
    ("uniform", 1000, 1, 1, 32),
    ("with_invalid", 500, 4, 16, 64),
    ("topk", 1024, 2, 8, 128),      # single-CTA path, full (2048 ids)
    ("topk", 1025, 2, 8, 128),      # crosses into the multi-CTA path
    ("topk", 4096, 2, 8, 128),      # multi-CTA, 8 chunks of 1024 (Mixtral T=4096)
    ("topk", 4097, 2, 8, 128),      # 8 chunks and a 2-id one
    ("skewed", 8192, 8, 128, 128),  # multi-CTA, Qwen3 T=8192
    ("topk", 8192, 8, 256, 128),    # multi-CTA, DeepSeek-V3 EP rank
    ("uniform", 16384, 2, 8, 256),
    ("with_invalid", 20000, 3, 1024, 16),
]


@pytest.mark.parametrize("kind,T,k,E,bm", SHAPES)
@pytest.mark.parametrize("dtype", [torch.int64, torch.int32])
def test_align_bit_exact(cuda_device, kind, T, k, E, bm, dtype):
    ids = gen_ids(kind, T, k, E, seed=T * 31 + E, dtype=dtype).to(cuda_device)
    run_and_compare(ids, E, bm)


def test_align_empty(cuda_device):
    run_and_compare(torch.zeros(0, 2, dtype=torch.int64, device=cuda_device), 8, 128)


@pytest.mark.parametrize("case", CASES, ids=lambda c: c.name)
def test_align_matches_reference_rows(cuda_device, case):
    """The reference's own per-expert row order (base.py:65-68)."""
    g = np.load(GOLDEN / f"{case.name}.npz")
    ids = torch.from_numpy(g["topk_ids"]).to(cuda_device)
    s, _, n = fm.moe_align_block_size(ids, 128, case.E)
    s = s.cpu().numpy()
    numel = ids.numel()
    got = s[s < numel]
    assert np.array_equal(got, g["expert_rows"])


def test_align_deterministic(cuda_device):
    ids = gen_ids("skewed", 8192, 8, 128, seed=7).to(cuda_device)
    a = fm.moe_align_block_size(ids, 128, 128)
    for _ in range(3):
        b = fm.moe_align_block_size(ids, 128, 128)
        for x, y in zip(a, b):
            assert torch.equal(x, y)
