"""Seeded input cases shared by the golden-fixture generator and the tests.

Each case regenerates its inputs from a CPU torch.Generator; the fixture
stores a SHA-256 of the regenerated tensors so that a drift of the generator
fails loudly instead of comparing unrelated data.
"""
from __future__ import annotations

import hashlib
from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class Case:
    name: str
    T: int
    H: int
    I: int
    E: int
    k: int
    dtype: torch.dtype
    seed: int
    weight_init: str = "fan_in"   # "fan_in": N(0, 1/fan_in); "ref": N(0, 0.02) as base.py:32-33
    bias_std: float = 0.0         # per-expert logit bias (skewed routing)
    renormalize: bool = True


CASES = [
    # base.py's own default shape (base.py:79-90) in three activation dtypes
    Case("toy_fp32", 83, 128, 64, 8, 2, torch.float32, 11, weight_init="ref"),
    Case("toy_bf16", 83, 128, 64, 8, 2, torch.bfloat16, 12, weight_init="ref"),
    Case("toy_fp16", 83, 128, 64, 8, 2, torch.float16, 13, weight_init="ref"),
    # the CPU-runnable fp32 configuration: H512 I1024 E8 top-2, T=64
    Case("cfg0_fp32", 64, 512, 1024, 8, 2, torch.float32, 21),
    # Qwen3-like routing (E=32 of 128 scaled down, top-8, biased logits)
    Case("qwen_mini_bf16", 37, 256, 128, 32, 8, torch.bfloat16, 31, bias_std=0.5),
    # DeepSeek-like routing (many experts, top-8)
    Case("dsv3_mini_fp32", 50, 256, 256, 64, 8, torch.float32, 41),
    # renormalize=False branch of base.py:46
    Case("norenorm_fp32", 20, 128, 64, 8, 2, torch.float32, 51, renormalize=False),
]

BY_NAME = {c.name: c for c in CASES}


def make_inputs(c: Case):
    """Returns (hidden [T,H] c.dtype, logits [T,E] f32, w1 [E,2I,H] f32, w2 [E,H,I] f32)."""
    g = torch.Generator().manual_seed(c.seed)
    hidden = torch.randn(c.T, c.H, generator=g).to(c.dtype)
    logits = torch.randn(c.T, c.E, generator=g)
    if c.bias_std:
        logits = logits + torch.randn(c.E, generator=g) * c.bias_std
    if c.weight_init == "ref":
        w1 = torch.randn(c.E, 2 * c.I, c.H, generator=g) * 0.02
        w2 = torch.randn(c.E, c.H, c.I, generator=g) * 0.02
    else:
        w1 = torch.randn(c.E, 2 * c.I, c.H, generator=g) / c.H ** 0.5
        w2 = torch.randn(c.E, c.H, c.I, generator=g) / c.I ** 0.5
    return hidden, logits, w1, w2


def digest(*tensors: torch.Tensor) -> str:
    h = hashlib.sha256()
    for t in tensors:
        h.update(t.contiguous().view(torch.uint8).numpy().tobytes())
    return h.hexdigest()


# ---------------------------------------------------------------------------
# Grouped top-k routing (kernels/track1-triton/groupedtopk/base.py)
# ---------------------------------------------------------------------------

@dataclass(frozen=True)
class GroupedCase:
    name: str
    T: int
    E: int
    topk: int
    renormalize: bool
    num_expert_group: int
    topk_group: int
    scoring_func: str
    routed_scaling_factor: float
    seed: int


GROUPED_CASES = [
    # the reference's default problem (groupedtopk/base.py:75-89)
    GroupedCase("gtk_default", 83, 256, 8, True, 8, 4, "softmax", 1.0, 61),
    # DeepSeek-V3-style: sigmoid scores, scaled weights
    GroupedCase("gtk_sigmoid_scaled", 64, 256, 8, True, 8, 4, "sigmoid", 2.5, 62),
    GroupedCase("gtk_norenorm", 50, 64, 6, False, 4, 2, "softmax", 1.0, 63),
    GroupedCase("gtk_one_group", 37, 32, 4, True, 4, 1, "sigmoid", 1.0, 64),
    GroupedCase("gtk_wide", 19, 1024, 16, True, 32, 8, "softmax", 1.0, 65),
]

GROUPED_BY_NAME = {c.name: c for c in GROUPED_CASES}


def make_grouped_inputs(c: GroupedCase):
    """Returns (hidden_states [T, 16] f16 (only its row count is used),
    gating_output [T, E] f32 ~ N(0, 1))."""
    g = torch.Generator().manual_seed(c.seed)
    hidden = torch.randn(c.T, 16, generator=g).to(torch.float16)
    logits = torch.randn(c.T, c.E, generator=g)
    return hidden, logits
