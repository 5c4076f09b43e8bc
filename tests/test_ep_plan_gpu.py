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
