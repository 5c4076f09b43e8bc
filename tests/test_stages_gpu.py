"""GPU: each stage of moe_fused_experts through its own C-ABI entry point,
against a plain torch fp32 computation of the same stage (the oracle's math
on the same rounded operands)."""
import ctypes

import pytest
import torch

from kernelswift_b200 import _lib
from kernelswift_b200 import fused_moe as fm
from oracle import moe_oracle as orc

pytestmark = pytest.mark.gpu


def p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def setup(T, H, I, E, k, seed, dtype=torch.bfloat16, dev="cuda"):
    g = torch.Generator().manual_seed(seed)
    hidden = torch.randn(T, H, generator=g).to(dtype)
    logits = torch.randn(T, E, generator=g)
    w1 = torch.randn(E, 2 * I, H, generator=g) / H ** 0.5
    w2 = torch.randn(E, H, I, generator=g) / I ** 0.5
    w, ids = orc.route(logits, k)
    return hidden.to(dev), w1.to(dev), w2.to(dev), w.to(dev), ids.to(dev)


def gathered(hidden, ids, E, k):
    sorted_ids, expert_ids, npp = fm.moe_align_block_size(ids, 128, E)
    L = sorted_ids.numel()
    numel = ids.numel()
    a = torch.zeros(L, hidden.shape[1], dtype=torch.bfloat16, device=hidden.device)
    _lib.call("moe_gather_rows", p(hidden), _lib.DT_BF16 if hidden.dtype == torch.bfloat16
              else _lib.DT_F32, hidden.shape[0], hidden.shape[1], k, p(sorted_ids), p(npp),
              L, numel, _lib.QUANT_NONE, p(a), _lib.DT_BF16, None, stream())
    return sorted_ids, expert_ids, npp, a


@pytest.mark.parametrize("T,H,E,k", [(5, 128, 8, 2), (300, 256, 16, 4)])
def test_gather(cuda_device, T, H, E, k):
    hidden, _, _, _, ids = setup(T, H, 64, E, k, seed=1)
    sorted_ids, _, npp, a = gathered(hidden, ids, E, k)
    s = sorted_ids.cpu()
    n = int(npp.item())
    numel = ids.numel()
    valid = (s[:n] < numel).nonzero().view(-1)
    want = hidden.cpu()[s[valid] // k]
    assert torch.equal(a.cpu()[valid], want)


GEMM_SHAPES = [
    # T, H, I, E, k, block_n
    (7, 128, 64, 8, 2, 0),
    (83, 128, 64, 8, 2, 128),
    (200, 512, 1024, 8, 2, 256),
    (64, 256, 128, 32, 8, 64),
    (333, 384, 224, 4, 2, 0),      # I = 224: down-GEMM K tail, gate-up N tile 64
]


@pytest.mark.parametrize("T,H,I,E,k,bn", GEMM_SHAPES)
def test_gate_up_gemm(cuda_device, T, H, I, E, k, bn):
    hidden, w1, w2, w, ids = setup(T, H, I, E, k, seed=T + H)
    sorted_ids, expert_ids, npp, a = gathered(hidden, ids, E, k)
    prep = fm.prepare_weights(w1, w2, "none", torch.bfloat16)
    L = sorted_ids.numel()
    act = torch.zeros(L, I, dtype=torch.bfloat16, device=cuda_device)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    _lib.call("moe_gemm_gate_up", _lib.QUANT_NONE, _lib.DT_BF16, p(a), None, p(prep.w13), None,
              p(sorted_ids), p(expert_ids), p(npp), L, ids.numel(), E, H, I, p(act), bn,
              p(status), stream())
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    s = sorted_ids.cpu()
    eids = expert_ids.cpu()
    n = int(npp.item())
    a_c, w1_c = a.cpu().float(), w1.cpu().to(torch.bfloat16).float()
    act_c = act.cpu().float()
    numel = ids.numel()
    for m in range(n):
        if s[m] >= numel:
            continue
        e = int(eids[m // 128])
        gu = a_c[m] @ w1_c[e].T
        ref = torch.nn.functional.silu(gu[:I]) * gu[I:]
        torch.testing.assert_close(act_c[m], ref, rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("T,H,I,E,k,bn", GEMM_SHAPES)
@pytest.mark.parametrize("splits", [1, 2])
def test_down_gemm_and_sum(cuda_device, T, H, I, E, k, bn, splits):
    hidden, w1, w2, w, ids = setup(T, H, I, E, k, seed=T + I)
    sorted_ids, expert_ids, npp, _ = gathered(hidden, ids, E, k)
    L = sorted_ids.numel()
    numel = ids.numel()
    g = torch.Generator().manual_seed(5)
    act = (torch.randn(L, I, generator=g) * 0.5).to(torch.bfloat16).to(cuda_device)
    prep = fm.prepare_weights(w1, w2, "none", torch.bfloat16)
    kb = -(-I * 2 // 128)
    if splits > kb:
        pytest.skip("fewer k-blocks than splits")
    part = torch.full((splits, numel, H), float("nan"), device=cuda_device)
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    _lib.call("moe_gemm_down", _lib.QUANT_NONE, _lib.DT_BF16, p(act), None, p(prep.w2), None,
              p(sorted_ids), p(expert_ids), p(npp), L, numel, E, H, I, p(w), _lib.DT_F32,
              splits, p(part), 0 if bn == 0 or H % bn else bn, p(status), stream())
    out = torch.empty(T, H, dtype=torch.float32, device=cuda_device)
    _lib.call("moe_sum_topk", p(part), splits, T, k, H, p(ids), _lib.DT_I64, E, p(out),
              _lib.DT_F32, stream())
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    s = sorted_ids.cpu()
    eids = expert_ids.cpu()
    act_c = act.cpu().float()
    w2_c = w2.cpu().to(torch.bfloat16).float()
    w_c = w.cpu().reshape(-1)
    ref_rows = torch.zeros(numel, H)
    for m in range(int(npp.item())):
        r = int(s[m])
        if r >= numel:
            continue
        e = int(eids[m // 128])
        ref_rows[r] = w_c[r] * (act_c[m] @ w2_c[e].T)
    got_rows = part.cpu().sum(0)
    torch.testing.assert_close(got_rows, ref_rows, rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(out.cpu(), ref_rows.view(T, k, H).sum(1), rtol=2e-2, atol=2e-2)


def test_prepare_regroup_and_cast(cuda_device):
    _, w1, w2, _, _ = setup(4, 128, 96, 3, 2, seed=9)
    prep = fm.prepare_weights(w1, w2, "none", torch.bfloat16)
    assert torch.equal(prep.w13.cpu(), orc.regroup_w13(w1.cpu()).to(torch.bfloat16))
    assert torch.equal(prep.w2.cpu(), w2.cpu().to(torch.bfloat16))


def test_prepare_int8_bit_exact(cuda_device):
    _, w1, w2, _, _ = setup(4, 256, 128, 4, 2, seed=10)
    prep = fm.prepare_weights(w1, w2, "int8")
    q1, s1 = orc.quant_int8_rows(w1.cpu())
    q2, s2 = orc.quant_int8_rows(w2.cpu())
    assert torch.equal(prep.w13.cpu(), orc.regroup_w13(q1.float()).to(torch.int8))
    assert torch.equal(prep.w13_scale.cpu(), orc.regroup_rows_vec(s1))
    assert torch.equal(prep.w2.cpu(), q2)
    assert torch.equal(prep.w2_scale.cpu(), s2)


def test_prepare_fp8_bit_exact(cuda_device):
    _, w1, w2, _, _ = setup(4, 256, 128, 4, 2, seed=11)
    prep = fm.prepare_weights(w1, w2, "fp8")
    q1, s1 = orc.quant_fp8_block(w1.cpu())
    q2, s2 = orc.quant_fp8_block(w2.cpu())
    assert torch.equal(prep.w13.cpu().view(torch.uint8),
                       orc.regroup_w13(q1.float()).to(torch.float8_e4m3fn).view(torch.uint8))
    assert torch.equal(prep.w13_scale.cpu(), s1)
    assert torch.equal(prep.w2.cpu().view(torch.uint8), q2.view(torch.uint8))
    assert torch.equal(prep.w2_scale.cpu(), s2)


def test_bounded_wait_reports_timeout(cuda_device):
    """A barrier nobody arrives on: the kernel gives up after the limit and
    reports MOE_ERR_TIMEOUT; the context stays usable."""
    status = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    _lib.call("moe_selftest_wait_timeout", p(status), 2000, stream())
    host = ctypes.c_int32(-1)
    _lib.call("moe_read_status", p(status), ctypes.byref(host), 1, stream())
    assert host.value == _lib.MOE_ERR_TIMEOUT
    assert int(status.item()) == 0  # reset
    x = torch.ones(16, device=cuda_device)
    assert float((x * 2).sum()) == 32.0


@pytest.mark.parametrize("quant", ["fp8", "int8"])
@pytest.mark.parametrize("H", [256, 7168, 320])
def test_gather_quantisers_bit_exact(cuda_device, quant, H):
    """The gather's per-token quantisation equals the oracle's activation
    quantiser bit for bit (fp8: per 128 columns, int8: per row)."""
    T, E, k = 37, 8, 2
    hidden, _, _, _, ids = setup(T, H, 64, E, k, seed=H)
    sorted_ids, expert_ids, npp = fm.moe_align_block_size(ids, 128, E)
    L = sorted_ids.numel()
    numel = ids.numel()
    if quant == "fp8":
        dst = torch.zeros(L, H, dtype=torch.uint8, device=cuda_device)
        scale = torch.zeros(L, -(-H // 128), device=cuda_device)
        code = _lib.QUANT_FP8_BLOCK
    else:
        dst = torch.zeros(L, H, dtype=torch.int8, device=cuda_device)
        scale = torch.zeros(L, device=cuda_device)
        code = _lib.QUANT_INT8_CHANNEL
    _lib.call("moe_gather_rows", p(hidden), _lib.DT_BF16, T, H, k, p(sorted_ids), p(npp), L,
              numel, code, p(dst), _lib.DT_E4M3 if quant == "fp8" else _lib.DT_I8, p(scale),
              stream())
    torch.cuda.synchronize()
    s = sorted_ids.cpu()
    n = int(npp.item())
    valid = (s[:n] < numel).nonzero().view(-1)
    rows = hidden.cpu()[s[valid] // k]
    if quant == "fp8":
        q, sc = orc.quant_fp8_group(rows)
        assert torch.equal(dst.cpu()[valid], q.view(torch.uint8))
    else:
        q, sc = orc.quant_int8_rows(rows, reciprocal=True)
        assert torch.equal(dst.cpu()[valid], q)
    assert torch.equal(scale.cpu()[valid], sc)


@pytest.mark.parametrize("T,k,E,world,invalid", [(4096, 2, 8, 2, False), (8192, 8, 256, 8, False),
                                                 (333, 4, 16, 4, True), (1, 8, 128, 8, False)])
def test_ep_plan_bit_exact(cuda_device, T, k, E, world, invalid):
    """moe_ep_plan equals the stable sort by destination rank (torch ops)."""
    from kernelswift_b200.ep import CudaBackend

    g = torch.Generator().manual_seed(T + E)
    ids = torch.topk(torch.randn(T, E, generator=g), k, dim=-1).indices
    if invalid:
        ids[::5, 0] = -1
        ids[1::7, -1] = E + 3
    order, send_eid, inv, counts = CudaBackend(None).plan(ids.to(cuda_device), E, world)
    flat = ids.reshape(-1)
    el = E // world
    valid = (flat >= 0) & (flat < E)
    dest = torch.where(valid, flat // el, torch.full_like(flat, world))
    want_order = torch.sort(dest, stable=True).indices
    want_counts = torch.bincount(dest, minlength=world + 1)
    n = int(want_counts[:world].sum())
    want_inv = torch.full_like(flat, -1)
    want_inv[want_order[:n]] = torch.arange(n)
    assert torch.equal(counts.cpu(), want_counts)
    assert torch.equal(order.cpu()[:n].long(), want_order[:n])
    assert torch.equal(send_eid.cpu()[:n].long(), (flat - dest * el)[want_order[:n]])
    assert torch.equal(inv.cpu().long(), want_inv)
