"""GPU: the decode path of moe_fused_experts (at most 16 routed rows, 16-bit
activations, unquantised weights: two weight-streaming kernels instead of the
align/gather/GEMM pipeline) against the fp32 oracle, with dropped slots,
int32/int64 ids, f32/bf16 weights and fp16 activations; the boundary with
the tensor-core path (17 routed rows); and moe_fused_moe (routing and
experts in one library call): bit-identical to fused_topk followed by
fused_experts."""
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

from kernelswift_b200 import fused_moe as fm
from oracle import moe_oracle as orc

pytestmark = pytest.mark.gpu

TOL = dict(rtol=2e-2, atol=2e-2)


def problem(T, H, I, E, k, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    hidden = torch.randn(T, H, generator=g).to(dtype)
    logits = torch.randn(T, E, generator=g)
    w1 = (torch.randn(E, 2 * I, H, generator=g) / H ** 0.5).to(dtype)
    w2 = (torch.randn(E, H, I, generator=g) / I ** 0.5).to(dtype)
    return hidden, logits, w1, w2


@pytest.mark.parametrize("T,H,I,E,k,dtype", [
    (1, 256, 128, 16, 8, torch.bfloat16),     # 8 routed rows (Qwen3-like top-8)
    (2, 256, 128, 16, 8, torch.bfloat16),     # 16: the largest decode problem
    (1, 512, 1024, 8, 2, torch.bfloat16),     # Mixtral-like top-2
    (5, 384, 256, 8, 2, torch.float16),
    (1, 128, 32, 4, 1, torch.bfloat16),       # smallest widths the planner takes
    (1, 2048, 768, 128, 8, torch.bfloat16),   # Qwen3-30B-A3B T=1
    (1, 256, 128, 32, 12, torch.bfloat16),    # 12 slots of one token
    (17, 256, 128, 16, 1, torch.bfloat16),    # 17 rows: tensor-core path
])
def test_decode_matches_oracle(cuda_device, T, H, I, E, k, dtype):
    hidden, logits, w1, w2 = problem(T, H, I, E, k, dtype, seed=T * 131 + H)
    w, ids = orc.route(logits, k)
    ref = orc.fused_experts(hidden, w1, w2, w, ids)
    prep = fm.prepare_weights(w1.to(cuda_device), w2.to(cuda_device), "none", dtype)
    for ids_dt, w_dt in ((torch.int32, torch.float32), (torch.int64, dtype)):
        out = fm.fused_experts(hidden.to(cuda_device), prep, None, w.to(w_dt).to(cuda_device),
                               ids.to(ids_dt).to(cuda_device))
        torch.testing.assert_close(out.float().cpu(), ref, **TOL)
        again = fm.fused_experts(hidden.to(cuda_device), prep, None,
                                 w.to(w_dt).to(cuda_device), ids.to(ids_dt).to(cuda_device))
        assert torch.equal(out, again)  # fixed reduction order


def test_decode_dropped_slots(cuda_device):
    T, H, I, E, k = 2, 256, 128, 8, 4
    hidden, logits, w1, w2 = problem(T, H, I, E, k, torch.bfloat16, seed=7)
    w, ids = orc.route(logits, k)
    ids[0, 1] = -1
    ids[1, 3] = E  # out of range: dropped
    keep = (ids >= 0) & (ids < E)
    ref = orc.fused_experts(hidden, w1, w2, w * keep, ids.clamp(0, E - 1))
    prep = fm.prepare_weights(w1.to(cuda_device), w2.to(cuda_device), "none", torch.bfloat16)
    out = fm.fused_experts(hidden.to(cuda_device), prep, None, w.to(cuda_device),
                           ids.to(torch.int32).to(cuda_device))
    torch.testing.assert_close(out.float().cpu(), ref, **TOL)


def test_decode_close_to_tensor_core_path(cuda_device, tmp_path):
    """The same problem with MOE_NO_DECODE_PATH=1 (align/gather/GEMMs) in a
    child process: the two paths agree within the bf16 tolerance."""
    T, H, I, E, k = 1, 512, 256, 16, 8
    code = f"""
import sys, torch
sys.path.insert(0, {str(Path(__file__).resolve().parent.parent)!r})
sys.path.insert(0, {str(Path(__file__).resolve().parent)!r})
from test_decode_gpu import run_case
torch.save(run_case(), {str(tmp_path / 'tc.pt')!r})
"""
    env = dict(os.environ, MOE_NO_DECODE_PATH="1")
    res = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True,
                         timeout=600)
    assert res.returncode == 0, res.stderr[-2000:]
    tc = torch.load(tmp_path / "tc.pt")
    dec = run_case()
    torch.testing.assert_close(dec.float(), tc.float(), **TOL)


def run_case():
    dev = torch.device("cuda", 0)
    T, H, I, E, k = 1, 512, 256, 16, 8
    hidden, logits, w1, w2 = problem(T, H, I, E, k, torch.bfloat16, seed=99)
    w, ids = orc.route(logits, k)
    prep = fm.prepare_weights(w1.to(dev), w2.to(dev), "none", torch.bfloat16)
    out = fm.fused_experts(hidden.to(dev), prep, None, w.to(dev), ids.to(torch.int32).to(dev))
    return out.cpu()


ROUTE_CASES = [
    # T, H, I, E, k, dtype, renormalize
    (1, 2048, 768, 128, 8, torch.bfloat16, True),    # Qwen3-30B-A3B T=1
    (2, 2048, 768, 128, 8, torch.bfloat16, True),    # 16 routed rows
    (1, 512, 1024, 8, 2, torch.float16, True),
    (3, 384, 256, 256, 4, torch.bfloat16, False),    # 256 experts, no renormalisation
    (8, 256, 128, 8, 1, torch.bfloat16, True),
    (1, 256, 128, 512, 8, torch.bfloat16, True),     # 512 experts
    (64, 512, 256, 16, 4, torch.bfloat16, True),     # tensor-core path
]


@pytest.mark.parametrize("T,H,I,E,k,dtype,renorm", ROUTE_CASES,
                         ids=[f"T{c[0]}_H{c[1]}_E{c[3]}_k{c[4]}" for c in ROUTE_CASES])
def test_fused_moe_equals_two_calls(cuda_device, T, H, I, E, k, dtype, renorm):
    """fused_moe (moe_fused_moe: routing inside the library call) writes the
    same ids and weights as fused_topk and the same output as fused_topk +
    fused_experts, bit for bit, and matches the oracle."""
    hidden, logits, w1, w2 = problem(T, H, I, E, k, dtype, seed=T * 7 + E)
    dev = cuda_device
    prep = fm.prepare_weights(w1.to(dev), w2.to(dev), "none", dtype)
    hd, ld = hidden.to(dev), logits.to(dev)
    w_ref, ids_ref = fm.fused_topk(hd, ld, k, renorm, weights_dtype=dtype)
    two = fm.fused_experts(hd, prep, None, w_ref, ids_ref)
    w_out = torch.full((T, k), -1.0, dtype=dtype, device=dev)
    ids_out = torch.full((T, k), -1, dtype=torch.int32, device=dev)
    one = fm.fused_experts(hd, prep, None, w_out, ids_out, router_logits=ld,
                           renormalize=renorm)
    torch.cuda.synchronize()
    assert torch.equal(ids_out, ids_ref) and torch.equal(w_out, w_ref)
    assert torch.equal(one, two)
    again = fm.fused_moe(hd, prep, None, ld, k, renorm)
    assert torch.equal(again, one)
    w, ids = orc.route(logits, k, renorm)
    assert torch.equal(ids_out.cpu().long(), ids)
    ref = orc.fused_experts(hidden, w1, w2, w, ids)
    torch.testing.assert_close(one.float().cpu(), ref, **TOL)


def test_fused_moe_bf16_logits_and_launch_count(cuda_device):
    """bf16 router logits route like fused_topk on them; the fused call's
    launch count is the routing kernel plus fused_experts' launches (fp32
    logits on the decode path: fused_experts' launches alone)."""
    T, H, I, E, k = 1, 2048, 768, 128, 8
    hidden, logits, w1, w2 = problem(T, H, I, E, k, torch.bfloat16, seed=5)
    dev = cuda_device
    prep = fm.prepare_weights(w1.to(dev), w2.to(dev), "none", torch.bfloat16)
    hd, lb = hidden.to(dev), logits.to(torch.bfloat16).to(dev)
    w_ref, ids_ref = fm.fused_topk(hd, lb, k, weights_dtype=torch.bfloat16)
    two = fm.fused_experts(hd, prep, None, w_ref, ids_ref)
    assert torch.equal(fm.fused_moe(hd, prep, None, lb, k), two)
    assert fm.fused_moe_launches(T, H, I, E, k, logits_dtype=torch.bfloat16) == 3
    assert fm.fused_moe_launches(T, H, I, E, k) == 2
    assert fm.fused_moe_launches(64, H, I, E, k) == 1 + fm.fused_experts_launches(64, H, I, E, k)


def test_modelnew_decode_graph_replay(cuda_device):
    """ModelNew at T=1 (routing kernel and the two decode kernels) captured in
    a CUDA graph: replays equal eager calls bit for bit."""
    T, H, I, E, k = 1, 2048, 768, 128, 8
    m = fm.ModelNew(E, k, H, I).to(cuda_device)
    g = torch.Generator(device=cuda_device).manual_seed(3)
    with torch.no_grad():
        m.w1.normal_(0, H ** -0.5, generator=g)
        m.w2.normal_(0, I ** -0.5, generator=g)
    cap = fm.CapturedMoE(m, T, H, E, dtype=torch.bfloat16, device=cuda_device)
    for seed in (1, 2, 3):
        gi = torch.Generator(device=cuda_device).manual_seed(seed)
        hidden = torch.randn(T, H, generator=gi, device=cuda_device).to(torch.bfloat16)
        logits = torch.randn(T, E, generator=gi, device=cuda_device)
        with torch.no_grad():
            eager = m(hidden, logits).clone()
        out = cap(hidden, logits)
        torch.cuda.synchronize()
        assert torch.equal(out, eager)
