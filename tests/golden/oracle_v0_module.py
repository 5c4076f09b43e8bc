"""v0 operator module for the device-timed v0/v1 runner: the fused-MoE
layer of kernels/track1-triton/fused_moe/base.py restated by the oracle
(oracle.moe_oracle.model_forward_native, base.py:35-76 op for op in the
activation dtype), with base.py's constructor, parameter names and default
problem (base.py:9-33, 79-90). Test infrastructure: it stands in for
base.py where the reference checkout is absent (the GPU box), so that
kernelswift_b200/ks_fused_moe.py can be compared with it through
kernelswift_b200.ab_runner exactly as auto_bench compares a v1 module with
base.py."""
import torch
import torch.nn as nn

from oracle import moe_oracle


class Model(nn.Module):
    def __init__(self, num_experts, top_k, hidden_size, intermediate_size, renormalize=True):
        super().__init__()
        self.top_k = top_k
        self.renormalize = renormalize
        self.w1 = nn.Parameter(torch.randn(num_experts, 2 * intermediate_size, hidden_size) * 0.02)
        self.w2 = nn.Parameter(torch.randn(num_experts, hidden_size, intermediate_size) * 0.02)

    def forward(self, hidden_states, router_logits):
        return moe_oracle.model_forward_native(hidden_states, router_logits, self.w1, self.w2,
                                               self.top_k, self.renormalize)


def get_inputs():
    num_tokens, hidden_size, num_experts = 83, 128, 8
    hidden_states = torch.randn(num_tokens, hidden_size, dtype=torch.float16, device="cuda")
    router_logits = torch.randn(num_tokens, num_experts, dtype=torch.float32, device="cuda")
    return [hidden_states, router_logits]


def get_init_inputs():
    return [8, 2, 128, 64]
