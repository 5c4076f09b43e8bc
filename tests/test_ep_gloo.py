"""CPU tests of the expert-parallel host logic over gloo ranks.

The exchange (split sizes, packing order, the three all_to_alls, the inverse
permutation of the combine) runs exactly as on GPUs; the device work is done
by a test-only CPU backend built on the oracle. A second test makes one rank
fail before its first collective and checks that the other rank's forward
ends with an error within the process group's timeout instead of hanging.
"""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import moe_oracle as orc


class CpuBackend:
    """Oracle-backed stand-in for CudaBackend (tests only)."""

    def __init__(self, w1_local, w2_local):
        self.w1, self.w2 = w1_local, w2_local

    def plan(self, topk_ids, num_experts, world):
        """moe_ep_plan restated with torch ops."""
        flat = topk_ids.reshape(-1).long()
        el = num_experts // world
        valid = (flat >= 0) & (flat < num_experts)
        dest = torch.where(valid, flat // el, torch.full_like(flat, world))
        order = torch.sort(dest, stable=True).indices
        counts = torch.bincount(dest, minlength=world + 1)
        n_send = int(counts[:world].sum())
        send_eid = (flat[order] - dest[order] * el).to(torch.int32)
        inv = torch.full_like(flat, -1)
        inv[order[:n_send]] = torch.arange(n_send)
        return order.to(torch.int32), send_eid, inv.to(torch.int32), counts

    def pack(self, hidden, order, top_k):
        return hidden[torch.div(order.long(), top_k, rounding_mode="floor")]

    def experts(self, rows, local_ids):
        ones = torch.ones(rows.shape[0], 1)
        return orc.fused_experts(rows, self.w1, self.w2, ones,
                                 local_ids.view(-1, 1).long()).to(rows.dtype)

    def combine(self, rows, inv, weights, num_tokens, top_k):
        w = weights.reshape(-1, 1).float()
        return (rows.float()[inv.long()] * w).view(num_tokens, top_k, -1).sum(1).to(rows.dtype)


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def problem(E, H, I, seed):
    g = torch.Generator().manual_seed(seed)
    w1 = torch.randn(E, 2 * I, H, generator=g) / H ** 0.5
    w2 = torch.randn(E, H, I, generator=g) / I ** 0.5
    return w1, w2


def worker(rank, world, port, E, k, T, H, I, fail_rank, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from kernelswift_b200.ep import ExpertParallelMoE

    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    try:
        w1, w2 = problem(E, H, I, seed=0)
        el = E // world
        g = torch.Generator().manual_seed(100 + rank)
        hidden = torch.randn(T + rank, H, generator=g)
        logits = torch.randn(T + rank, E, generator=g)
        w, ids = orc.route(logits, k)
        ep = ExpertParallelMoE(None, None, E, k,
                               backend=CpuBackend(w1[rank * el:(rank + 1) * el],
                                                  w2[rank * el:(rank + 1) * el]))
        if rank == fail_rank:
            raise RuntimeError("planted failure before the first collective")
        out = ep(hidden, w, ids)
        ref = orc.fused_experts(hidden, w1, w2, w, ids)
        err = float((out - ref).abs().max())
        result_q.put((rank, "ok", err))
    except Exception as exc:  # reported to the parent
        result_q.put((rank, "error", repr(exc)[:200]))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def run(world, fail_rank=-1, E=8, k=2, T=37, H=64, I=32):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=worker, args=(r, world, port, E, k, T, H, I, fail_rank, q))
             for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, status, info = q.get(timeout=120)
        results[rank] = (status, info)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return results


@pytest.mark.parametrize("world,E,k", [(2, 8, 2), (4, 16, 4)])
def test_ep_matches_oracle(world, E, k):
    res = run(world, E=E, k=k)
    for rank in range(world):
        status, info = res[rank]
        assert status == "ok", (rank, info)
        assert info < 1e-4, (rank, info)


def test_ep_rank_failure_surfaces_as_error():
    res = run(2, fail_rank=1)
    assert res[1][0] == "error" and "planted failure" in res[1][1]
    # the surviving rank's first collective must fail, not hang
    assert res[0][0] == "error", res[0]
