"""GPU: the expert-parallel dispatch plan over many CTAs (moe_ep_plan_ws,
more than 8192 slots) against the single-CTA plan (moe_ep_plan) bit for
bit, and against a CPU restatement, for several rank counts, int32/int64
ids and ids outside [0, E). The plan is a pure function of the ids, so one
GPU covers any rank count.
"""
import ctypes
import os

import pytest
import torch

from kernelswift_b200 import _lib

pytestmark = pytest.mark.gpu


def p(t):
    return ctypes.c_void_p(t.data_ptr())


def stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def plan(ids, E, world, multi):
    n = ids.numel()
    dev = ids.device
    order = torch.full((n,), -7, dtype=torch.int32, device=dev)
    send_eid = torch.full((n,), -7, dtype=torch.int32, device=dev)
    inv = torch.full((n,), -7, dtype=torch.int32, device=dev)
    counts = torch.zeros(world + 1, dtype=torch.int64, device=dev)
    code = _lib.DT_I32 if ids.dtype == torch.int32 else _lib.DT_I64
    if multi:
        nbytes = ctypes.c_size_t(0)
        _lib.call("moe_ep_plan_workspace_size", n, world, ctypes.byref(nbytes))
        ws = torch.empty(max(nbytes.value, 16), dtype=torch.uint8, device=dev)
        _lib.call("moe_ep_plan_ws", p(ids), code, n, E, world, p(order), p(send_eid), p(inv),
                  p(counts), p(ws), ws.numel(), stream())
    else:
        _lib.call("moe_ep_plan", p(ids), code, n, E, world, p(order), p(send_eid), p(inv),
                  p(counts), stream())
    torch.cuda.synchronize()
    n_send = int(counts[:world].sum())
    return order[:n_send].cpu(), send_eid[:n_send].cpu(), inv.cpu(), counts.cpu()


def cpu_plan(ids, E, world):
    flat = ids.reshape(-1).long().cpu()
    el = E // world
    valid = (flat >= 0) & (flat < E)
    dest = torch.where(valid, flat // el, torch.full_like(flat, world))
    order = torch.sort(dest, stable=True).indices
    counts = torch.bincount(dest, minlength=world + 1)
    n_send = int(counts[:world].sum())
    send_eid = (flat[order] - dest[order] * el)[:n_send].to(torch.int32)
    inv = torch.full_like(flat, -1)
    inv[order[:n_send]] = torch.arange(n_send)
    return order[:n_send].to(torch.int32), send_eid, inv.to(torch.int32), counts


@pytest.mark.parametrize("numel,E,world", [(8193, 8, 2), (20000, 16, 4), (65536, 256, 8),
                                           (300000, 256, 32), (100000, 128, 128),
                                           (50000, 8, 1)])
@pytest.mark.parametrize("dtype", [torch.int32, torch.int64])
def test_multi_cta_plan_matches_single_cta_and_cpu(cuda_device, numel, E, world, dtype):
    g = torch.Generator().manual_seed(numel + world)
    ids = torch.randint(0, E, (numel,), generator=g)
    ids[::97] = -1   # dropped slots
    ids[5::131] = E  # out of range
    ids = ids.to(dtype).to(cuda_device)
    multi = plan(ids, E, world, True)
    single = plan(ids, E, world, False)
    for a, b in zip(multi, single):
        assert torch.equal(a, b)
    for a, b in zip(multi, cpu_plan(ids, E, world)):
        assert torch.equal(a.long(), b.long())


@pytest.mark.parametrize("T,E,k,world", [(37, 8, 2, 2), (8192, 256, 8, 8), (4096, 128, 8, 4),
                                         (5000, 64, 4, 32), (1, 16, 4, 1), (3000, 8, 2, 8)])
@pytest.mark.parametrize("dtype", [torch.int32, torch.int64])
def test_dedup_plan_kernel_matches_torch(cuda_device, T, E, k, world, dtype):
    """moe_ep_plan_dedup equals ep.dedup_plan (the torch restatement) bit for
    bit: send rows, local ids, weights, inverse table and counts, with
    dropped and out-of-range ids."""
    from kernelswift_b200.ep import CudaBackend, dedup_plan
    from oracle import moe_oracle as orc

    g = torch.Generator().manual_seed(T + world)
    w, ids = orc.route(torch.randn(T, E, generator=g) + torch.linspace(0, 1, E), k)
    if T > 10:
        ids[3, 0] = -1
        ids[7, k - 1] = E
    wb = w.to(torch.bfloat16)  # weights in the activation dtype, as the model passes them
    ref = dedup_plan(ids, wb, E, world)
    got = CudaBackend(None).plan_dedup(ids.to(dtype).to(cuda_device), wb.to(cuda_device), E,
                                       world)
    torch.cuda.synchronize()
    n = int(ref[4][:world].sum())
    tokens, eid, sw, inv, counts = (x.cpu() for x in got)
    assert torch.equal(counts, ref[4].cpu())
    assert torch.equal(tokens[:n], ref[0].cpu())
    assert torch.equal(eid[:n], ref[1].cpu())
    assert torch.equal(sw[:n], ref[2].cpu())
    assert torch.equal(inv, ref[3].cpu())


def test_num_tokens_dev_bounds_the_expert_pass(cuda_device):
    """fused_experts with a device-side token count: rows below the count
    equal a plain call on those tokens bit for bit; rows past it are not
    written (their NaN sentinel survives)."""
    from kernelswift_b200 import fused_moe as fm
    from oracle import moe_oracle as orc

    T, H, I, E, k, n = 3000, 256, 512, 16, 4, 1234
    g = torch.Generator().manual_seed(4)
    hidden = torch.randn(T, H, generator=g).to(torch.bfloat16).to(cuda_device)
    w, ids = orc.route(torch.randn(T, E, generator=g), k)
    w, ids = w.to(cuda_device), ids.to(torch.int32).to(cuda_device)
    w1 = (torch.randn(E, 2 * I, H, generator=g) / H ** 0.5).to(cuda_device)
    w2 = (torch.randn(E, H, I, generator=g) / I ** 0.5).to(cuda_device)
    prep = fm.prepare_weights(w1, w2, "none", torch.bfloat16)
    ids_junk = ids.clone()
    ids_junk[n:] = 0  # present but past the count: must be ignored
    count = torch.tensor([n], dtype=torch.int32, device=cuda_device)
    out = torch.full_like(hidden, float("nan"))
    fm.fused_experts(hidden, prep, None, w, ids_junk, out=out, num_tokens_dev=count)
    ref = fm.fused_experts(hidden[:n].contiguous(), prep, None, w[:n].contiguous(),
                           ids[:n].contiguous())
    torch.cuda.synchronize()
    assert torch.equal(out[:n], ref)
    assert bool(torch.isnan(out[n:]).all())
