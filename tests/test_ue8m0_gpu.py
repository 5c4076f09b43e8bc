"""GPU: the fp8 path with power-of-two (UE8M0) block scales applied by the
tensor core (quant "fp8-ue8m0", moe_grouped_gemm_mx_kernel).

  - weight preparation: e4m3 bytes and scale-factor images bit-exact with the
    oracle's quantiser and image layout;
  - activation gather: e4m3 rows and image bytes bit-exact for every routed
    row;
  - the whole layer: relative L2 <= 5e-2 against the fp32 dequantised oracle,
    both N tiles, K-split and dropped slots, deterministic repeats;
  - the tensor-memory layout of one scale-factor chunk copy on its own.
"""
import ctypes

import pytest
import torch

from kernelswift_b200 import _lib
from kernelswift_b200 import fused_moe as fm
from oracle import moe_oracle as orc
from sampled import cover_tokens, oracle_on_tokens

pytestmark = pytest.mark.gpu

REL_L2 = 5e-2


def p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def weights(E, H, I, seed, dev):
    """N(0, 1/fan_in) expert weights drawn on the device (the DeepSeek-V3
    shape is 45 GB of fp32)."""
    g = torch.Generator(device=dev).manual_seed(seed)
    w1 = torch.randn(E, 2 * I, H, generator=g, device=dev) / H ** 0.5
    w2 = torch.randn(E, H, I, generator=g, device=dev) / I ** 0.5
    return w1, w2


def expected_row_bytes(block_bytes, rows_total, regroup):
    """Per-row scale bytes [E, R, KB] of a prepared weight: each row carries
    its 128x128 block's byte, rows of w13 in the regrouped order."""
    per_row = block_bytes.repeat_interleave(128, dim=1)[:, :rows_total]
    return orc.regroup_w13(per_row) if regroup else per_row


def test_scale_factor_copy_layout(cuda_device):
    """tcgen05.cp 32x128b.warpx4 of one chunk: lane l, column c holds word
    4 * (l % 32) + c, in all four 32-lane quarters."""
    g = torch.Generator().manual_seed(0)
    chunk = torch.randint(0, 2 ** 31 - 1, (128,), generator=g, dtype=torch.int64)
    chunk_dev = chunk.to(torch.int32).to(cuda_device)
    out = torch.zeros(128 * 4, dtype=torch.int32, device=cuda_device)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    _lib.call("moe_selftest_sf_copy", p(chunk_dev), p(out), p(status), stream())
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    lanes = torch.arange(128).unsqueeze(1)
    cols = torch.arange(4).unsqueeze(0)
    want = chunk.to(torch.int32)[4 * (lanes % 32) + cols]
    assert torch.equal(out.cpu().view(128, 4), want)


@pytest.mark.parametrize("E,H,I", [(4, 256, 128), (3, 384, 256)])
def test_prepare_matches_oracle(cuda_device, E, H, I):
    w1, w2 = weights(E, H, I, seed=E * H, dev=cuda_device)
    prep = fm.prepare_weights(w1, w2, "fp8-ue8m0")
    torch.cuda.synchronize()
    q1, b1 = orc.quant_fp8_block_ue8m0(w1.cpu())
    q2, b2 = orc.quant_fp8_block_ue8m0(w2.cpu())
    assert torch.equal(prep.w13.cpu().view(torch.uint8), orc.regroup_w13(q1).view(torch.uint8))
    assert torch.equal(prep.w2.cpu().view(torch.uint8), q2.view(torch.uint8))
    got13 = orc.sf_image_decode(prep.w13_scale, E, 2 * I, H // 128)
    got2 = orc.sf_image_decode(prep.w2_scale, E, H, I // 128)
    assert torch.equal(got13, expected_row_bytes(b1, 2 * I, True))
    assert torch.equal(got2, expected_row_bytes(b2, H, False))


@pytest.mark.parametrize("T,H,E,k", [(5, 128, 8, 2), (300, 640, 16, 4)])
def test_gather_matches_oracle(cuda_device, T, H, E, k):
    g = torch.Generator().manual_seed(T)
    hidden = (torch.randn(T, H, generator=g) * 2).to(torch.bfloat16).to(cuda_device)
    hidden[1] = 0  # an all-zero row
    _, ids = orc.route(torch.randn(T, E, generator=g), k)
    ids = ids.to(cuda_device)
    sorted_ids, _, npp = fm.moe_align_block_size(ids, 128, E)
    L = sorted_ids.numel()
    a = torch.zeros(L, H, dtype=torch.uint8, device=cuda_device)
    img = torch.zeros(_lib.load().moe_ue8m0_scale_bytes(1, L, H), dtype=torch.uint8,
                      device=cuda_device)
    _lib.call("moe_gather_rows", p(hidden), _lib.DT_BF16, T, H, k, p(sorted_ids), p(npp), L,
              ids.numel(), _lib.QUANT_FP8_UE8M0, p(a), _lib.DT_E4M3, p(img), stream())
    torch.cuda.synchronize()
    s = sorted_ids.cpu()
    n = int(npp.item())
    valid = (s[:n] < ids.numel()).nonzero().view(-1)
    q, b = orc.quant_fp8_group_ue8m0(hidden.cpu()[s[valid] // k])
    assert torch.equal(a.cpu()[valid], q.view(torch.uint8))
    got = orc.sf_image_decode(img, 1, L, H // 128)[0]
    assert torch.equal(got[valid], b)


def oracle_rows(hidden, w1, w2, w, ids, tokens):
    sub = ids[tokens]
    hit = torch.unique(sub[(sub >= 0) & (sub < w1.shape[0])])
    remap = torch.full((w1.shape[0] + 1,), -1, dtype=torch.int64)
    remap[hit] = torch.arange(hit.numel())
    sub = torch.where((sub >= 0) & (sub < w1.shape[0]), sub, torch.full_like(sub, w1.shape[0]))
    keep = remap[sub] >= 0
    return orc.fused_experts_fp8_ue8m0(hidden[tokens].cpu().float(), w1[hit].cpu(),
                                       w2[hit].cpu(), w[tokens] * keep,
                                       remap[sub].clamp_min(0))


LAYER_SHAPES = [
    # name, T, H, I, E, k, tokens checked
    ("small", 50, 256, 256, 16, 4, 50),
    ("decode_T1", 1, 512, 256, 32, 8, 1),     # K-split down GEMM
    ("tail_blocks", 129, 384, 128, 8, 2, 129),
    ("wide", 700, 1024, 512, 8, 2, 64),       # 256-wide tiles
    ("dsv3_T64", 64, 7168, 2048, 256, 8, 64),
    # DeepSeek-V3 at T=4096: the first token of every hit expert + 32 more
    ("dsv3_T4096", 4096, 7168, 2048, 256, 8, -32),
]


@pytest.mark.parametrize("name,T,H,I,E,k,n_check", LAYER_SHAPES, ids=[s[0] for s in LAYER_SHAPES])
def test_layer_matches_oracle(cuda_device, name, T, H, I, E, k, n_check):
    w1, w2 = weights(E, H, I, seed=T + H, dev=cuda_device)
    g = torch.Generator().manual_seed(T + 1)
    hidden = torch.randn(T, H, generator=g).to(torch.bfloat16).to(cuda_device)
    w, ids = orc.route(torch.randn(T, E, generator=g), k)
    prep = fm.prepare_weights(w1, w2, "fp8-ue8m0")
    out = fm.fused_experts(hidden, prep, None, w.to(cuda_device), ids.to(cuda_device),
                           use_fp8_w8a8=True)
    again = fm.fused_experts(hidden, prep, None, w.to(cuda_device), ids.to(cuda_device),
                             use_fp8_w8a8=True)
    torch.cuda.synchronize()
    assert torch.equal(out, again)
    if n_check < 0:  # every hit expert, plus -n_check random tokens
        tokens = cover_tokens(ids, -n_check)
        ref = oracle_on_tokens("fp8-ue8m0", hidden, w1, w2, w, ids, tokens)
    else:
        tokens = torch.randperm(T, generator=torch.Generator().manual_seed(0))[:n_check]
        ref = oracle_rows(hidden, w1, w2, w, ids, tokens)
    assert orc.rel_l2(out.cpu()[tokens], ref) <= REL_L2


def test_dropped_slots_and_int64_ids(cuda_device):
    T, H, I, E, k = 40, 256, 256, 8, 4
    w1, w2 = weights(E, H, I, seed=11, dev=cuda_device)
    g = torch.Generator().manual_seed(12)
    hidden = torch.randn(T, H, generator=g).to(torch.bfloat16).to(cuda_device)
    w, ids = orc.route(torch.randn(T, E, generator=g), k)
    ids[3, 1] = -1
    ids[7, 0] = E
    out = fm.fused_experts(hidden, w1, w2, w.to(cuda_device), ids.to(cuda_device),
                           use_fp8_w8a8=True, scale_format="ue8m0")
    torch.cuda.synchronize()
    ref = oracle_rows(hidden, w1, w2, w, ids, torch.arange(T))
    assert orc.rel_l2(out.cpu(), ref) <= REL_L2


def test_both_tile_widths_agree(cuda_device):
    """moe_gemm_gate_up with 128- and 256-wide tiles writes the same
    activations (each tile's accumulation order over K is the same)."""
    T, H, I, E, k = 200, 512, 256, 8, 2
    w1, w2 = weights(E, H, I, seed=5, dev=cuda_device)
    prep = fm.prepare_weights(w1, w2, "fp8-ue8m0")
    g = torch.Generator().manual_seed(6)
    hidden = torch.randn(T, H, generator=g).to(torch.bfloat16).to(cuda_device)
    _, ids = orc.route(torch.randn(T, E, generator=g), k)
    ids = ids.to(cuda_device)
    sorted_ids, expert_ids, npp = fm.moe_align_block_size(ids, 128, E)
    L = sorted_ids.numel()
    a = torch.zeros(L, H, dtype=torch.uint8, device=cuda_device)
    img = torch.zeros(_lib.load().moe_ue8m0_scale_bytes(1, L, H), dtype=torch.uint8,
                      device=cuda_device)
    _lib.call("moe_gather_rows", p(hidden), _lib.DT_BF16, T, H, k, p(sorted_ids), p(npp), L,
              ids.numel(), _lib.QUANT_FP8_UE8M0, p(a), _lib.DT_E4M3, p(img), stream())
    acts = []
    for bn in (128, 256):
        act = torch.zeros(L, I, dtype=torch.bfloat16, device=cuda_device)
        _lib.call("moe_gemm_gate_up", _lib.QUANT_FP8_UE8M0, _lib.DT_BF16, p(a), p(img),
                  p(prep.w13), p(prep.w13_scale), p(sorted_ids), p(expert_ids), p(npp), L,
                  ids.numel(), E, H, I, p(act), bn, None, stream())
        acts.append(act)
    torch.cuda.synchronize()
    s = sorted_ids.cpu()
    n = int(npp.item())
    valid = (s[:n] < ids.numel()).nonzero().view(-1)
    assert torch.equal(acts[0].cpu()[valid], acts[1].cpu()[valid])


def test_default_fp8_recipe(cuda_device):
    """use_fp8_w8a8 without a scale format: unquantised weights take the
    power-of-two recipe (bit-identical to scale_format="ue8m0"); weights
    given as e4m3 with fp32 block scales take the absmax / 448 kernel."""
    T, H, I, E, k = 60, 256, 256, 8, 2
    w1, w2 = weights(E, H, I, seed=21, dev=cuda_device)
    g = torch.Generator().manual_seed(22)
    hidden = torch.randn(T, H, generator=g).to(torch.bfloat16).to(cuda_device)
    w, ids = orc.route(torch.randn(T, E, generator=g), k)
    w, ids = w.to(cuda_device), ids.to(cuda_device)
    default = fm.fused_experts(hidden, w1, w2, w, ids, use_fp8_w8a8=True).clone()
    mx = fm.fused_experts(hidden, w1, w2, w, ids, use_fp8_w8a8=True, scale_format="ue8m0")
    assert torch.equal(default, mx)
    q1, s1 = orc.quant_fp8_block(w1.cpu())
    q2, s2 = orc.quant_fp8_block(w2.cpu())
    pre = fm.fused_experts(hidden, q1.to(cuda_device), q2.to(cuda_device), w, ids,
                           use_fp8_w8a8=True, w1_scale=s1.to(cuda_device),
                           w2_scale=s2.to(cuda_device)).clone()
    f32 = fm.fused_experts(hidden, w1, w2, w, ids, use_fp8_w8a8=True, scale_format="fp32")
    assert torch.equal(pre, f32)
