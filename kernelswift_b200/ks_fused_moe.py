"""auto_bench.py v1 module of the B200 fused-MoE operator.

Usage (with this repository on PYTHONPATH, on a B200):

    PYTHONPATH=/path/to/repo python auto_bench.py \\
        --v0_file kernels/track1-triton/fused_moe/base.py \\
        --v1_file /path/to/repo/kernelswift_b200/ks_fused_moe.py

auto_bench keeps only imports, function/class definitions and literal
assignments of this file (auto_bench.py:100-124), so everything lives behind
the import below. get_inputs/get_init_inputs return the reference's default
problem (T=83, H=128, E=8, top-2, I=64, fp16 hidden, fp32 logits); the harness
feeds the v0 module's inputs to both models anyway (auto_bench.py:654).
"""
import torch

from kernelswift_b200.fused_moe import ModelNew  # noqa: F401


def get_inputs():
    num_tokens, hidden_size, num_experts = 83, 128, 8
    hidden_states = torch.randn(num_tokens, hidden_size, dtype=torch.float16, device="cuda")
    router_logits = torch.randn(num_tokens, num_experts, dtype=torch.float32, device="cuda")
    return [hidden_states, router_logits]


def get_init_inputs():
    # num_experts, top_k, hidden_size, intermediate_size
    return [8, 2, 128, 64]
