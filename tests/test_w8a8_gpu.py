"""GPU: fp8 block-scaled (scale = absmax / 448, scale_format "fp32") and
int8 per-channel W8A8 paths against the fp32 dequantised oracle (relative
L2 <= 5e-2). The power-of-two scale recipe has its own tests
(test_ue8m0_gpu.py)."""
import pytest
import torch

from kernelswift_b200 import fused_moe as fm
from oracle import moe_oracle as orc
from sampled import cover_tokens, oracle_on_tokens

pytestmark = pytest.mark.gpu

REL_L2 = 5e-2


def problem(T, H, I, E, k, seed, bias=0.0, device="cuda"):
    g = torch.Generator().manual_seed(seed)
    hidden = torch.randn(T, H, generator=g).to(torch.bfloat16)
    logits = torch.randn(T, E, generator=g)
    if bias:
        logits = logits + torch.randn(E, generator=g) * bias
    w, ids = orc.route(logits, k)
    gd = torch.Generator(device=device).manual_seed(seed)
    w1 = torch.randn(E, 2 * I, H, generator=gd, device=device) / H ** 0.5
    w2 = torch.randn(E, H, I, generator=gd, device=device) / I ** 0.5
    return hidden.to(device), w1, w2, w, ids


# DeepSeek-V3 (H=7168, I=2048, E=256, top-8) fp8 at T in {64, 4096}; the
# Qwen3-30B-A3B shape (H=2048, I=768, E=128, top-8, skewed routing) in int8
# at T in {1, 64, 1024, 8192}. Up to 64 tokens every token is checked;
# above, the first token of every hit expert plus `extra` random tokens, so
# every expert's weights and scales that the batch uses are compared.
FP8_SHAPES = [
    # name, T, H, I, E, k, extra random tokens
    ("small", 50, 256, 256, 16, 4, 0),
    ("tail_blocks", 129, 384, 128, 8, 2, 129),
    ("dsv3_T64", 64, 7168, 2048, 256, 8, 0),
    ("dsv3_T4096", 4096, 7168, 2048, 256, 8, 32),
]


def check_tokens(T, ids, extra):
    return torch.arange(T) if T <= 64 else cover_tokens(ids, extra)


@pytest.mark.parametrize("name,T,H,I,E,k,extra", FP8_SHAPES, ids=[s[0] for s in FP8_SHAPES])
def test_fp8_block_w8a8(cuda_device, name, T, H, I, E, k, extra):
    hidden, w1, w2, w, ids = problem(T, H, I, E, k, seed=T + H)
    out = fm.fused_experts(hidden, w1, w2, w.to(cuda_device), ids.to(cuda_device),
                           use_fp8_w8a8=True, block_shape=[128, 128], scale_format="fp32")
    torch.cuda.synchronize()
    tokens = check_tokens(T, ids, extra)
    ref = oracle_on_tokens("fp8", hidden, w1, w2, w, ids, tokens)
    assert orc.rel_l2(out.cpu()[tokens], ref) <= REL_L2


INT8_SHAPES = [
    ("small", 50, 256, 256, 16, 4, 0),
    ("qwen3_T1", 1, 2048, 768, 128, 8, 0),
    ("qwen3_T64", 64, 2048, 768, 128, 8, 0),
    ("qwen3_T1024", 1024, 2048, 768, 128, 8, 32),
    ("qwen3_T8192", 8192, 2048, 768, 128, 8, 64),
]


@pytest.mark.parametrize("name,T,H,I,E,k,extra", INT8_SHAPES, ids=[s[0] for s in INT8_SHAPES])
def test_int8_channel_w8a8(cuda_device, name, T, H, I, E, k, extra):
    hidden, w1, w2, w, ids = problem(T, H, I, E, k, seed=T + 7, bias=0.5)
    out = fm.fused_experts(hidden, w1, w2, w.to(cuda_device), ids.to(cuda_device),
                           use_int8_w8a8=True)
    torch.cuda.synchronize()
    tokens = check_tokens(T, ids, extra)
    ref = oracle_on_tokens("int8", hidden, w1, w2, w, ids, tokens)
    assert orc.rel_l2(out.cpu()[tokens], ref) <= REL_L2


def test_fp8_prequantised_weights_pass_through(cuda_device):
    """Already-e4m3 weights with their block scales give the same result as
    quantising the fp32 weights inside prepare_weights."""
    hidden, w1, w2, w, ids = problem(40, 256, 256, 8, 2, seed=3)
    q1, s1 = orc.quant_fp8_block(w1.cpu())
    q2, s2 = orc.quant_fp8_block(w2.cpu())
    a = fm.fused_experts(hidden, w1, w2, w.to(cuda_device), ids.to(cuda_device),
                         use_fp8_w8a8=True, scale_format="fp32").clone()
    b = fm.fused_experts(hidden, q1.to(cuda_device), q2.to(cuda_device), w.to(cuda_device),
                         ids.to(cuda_device), use_fp8_w8a8=True, w1_scale=s1.to(cuda_device),
                         w2_scale=s2.to(cuda_device))
    assert torch.equal(a, b)
