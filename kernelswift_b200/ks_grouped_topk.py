"""auto_bench.py v1 module of the B200 grouped top-k routing kernel.

Usage (with this repository on PYTHONPATH, on a B200):

    PYTHONPATH=/path/to/repo python auto_bench.py \\
        --v0_file kernels/track1-triton/groupedtopk/base.py \\
        --v1_file /path/to/repo/kernelswift_b200/ks_grouped_topk.py

get_inputs/get_init_inputs return the reference's default problem
(groupedtopk/base.py:75-89: 83 tokens, 256 experts in 8 groups, top-4
groups, top-8, renormalised).
"""
import torch

from kernelswift_b200.fused_moe import GroupedTopK as ModelNew  # noqa: F401


def get_inputs():
    num_tokens, hidden_size, num_experts = 83, 7168, 256
    hidden_states = torch.randn(num_tokens, hidden_size, dtype=torch.float16, device="cuda")
    gating_output = torch.randn(num_tokens, num_experts, dtype=torch.float32, device="cuda")
    return [hidden_states, gating_output]


def get_init_inputs():
    # topk, renormalize, num_expert_group, topk_group
    return [8, True, 8, 4]
