"""CPU tests of the expert-parallel host logic over gloo ranks.

The exchange (split sizes, packing order, the three all_to_alls, the inverse
permutation of the combine) runs exactly as on GPUs; the device work is done
by a test-only CPU backend built on the oracle. The deduplicated exchange
(one row per token and destination rank) runs its torch plan unchanged, in
one piece and pipelined in token chunks (async all_to_alls, one chunk's
transfer in flight during the previous chunk's experts). A second test
makes one rank
fail before its first collective and checks that the other rank's forward
ends with an error within the process group's timeout instead of hanging. A
third replays the peer-memory exchange's placement rule (deduplicated
rows, counts matrix, destination offsets, the receiver's row count, combine
addressing) on 2 and 4 ranks with uneven token counts.
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

    def experts_weighted(self, rows, local_ids, weights):
        """sum_j w_j * expert_j(row), slots with id -1 dropped."""
        keep = local_ids >= 0
        return orc.fused_experts(rows, self.w1, self.w2, weights * keep,
                                 local_ids.long().clamp_min(0)).to(rows.dtype)

    def combine(self, rows, inv, weights, num_tokens, top_k):
        """moe_combine_rows: slots with inv < 0 contribute nothing."""
        inv = inv.long()
        w = (weights.reshape(-1).float() * (inv >= 0)).unsqueeze(1)
        if rows.shape[0] == 0:
            return torch.zeros(num_tokens, rows.shape[1], dtype=rows.dtype)
        picked = rows.float()[inv.clamp_min(0)] * w
        return picked.view(num_tokens, top_k, -1).sum(1).to(rows.dtype)


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def problem(E, H, I, seed):
    g = torch.Generator().manual_seed(seed)
    w1 = torch.randn(E, 2 * I, H, generator=g) / H ** 0.5
    w2 = torch.randn(E, H, I, generator=g) / I ** 0.5
    return w1, w2


def worker(rank, world, port, E, k, T, H, I, fail_rank, result_q, dedup=False, chunks=1):
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
                                                  w2[rank * el:(rank + 1) * el]),
                               dedup=dedup, chunks=chunks)
        if rank == fail_rank:
            raise RuntimeError("planted failure before the first collective")
        out = ep(hidden, w, ids)
        ref = orc.fused_experts(hidden, w1, w2, w, ids)
        err = float((out - ref).abs().max())
        if dedup or chunks > 1:
            # rows received = (token, rank) pairs routed here, over all senders
            sent = torch.tensor([len({int(e) // el for e in row}) for row in ids])
            n = torch.tensor([int(sent.sum()), ep.last_rows_received])
            dist.all_reduce(n)
            if int(n[0]) != int(n[1]):
                raise AssertionError(f"rows sent {int(n[0])} != rows received {int(n[1])}")
        result_q.put((rank, "ok", err))
    except Exception as exc:  # reported to the parent
        result_q.put((rank, "error", repr(exc)[:200]))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def run(world, fail_rank=-1, E=8, k=2, T=37, H=64, I=32, dedup=False, chunks=1):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=worker,
                         args=(r, world, port, E, k, T, H, I, fail_rank, q, dedup, chunks))
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


@pytest.mark.parametrize("world,E,k", [(2, 8, 2), (4, 16, 4), (8, 16, 2)])
def test_ep_matches_oracle(world, E, k):
    res = run(world, E=E, k=k)
    for rank in range(world):
        status, info = res[rank]
        assert status == "ok", (rank, info)
        assert info < 1e-4, (rank, info)


@pytest.mark.parametrize("world,E,k", [(2, 8, 2), (4, 16, 4), (8, 32, 8)])
def test_ep_dedup_matches_oracle(world, E, k):
    res = run(world, E=E, k=k, dedup=True)
    for rank in range(world):
        status, info = res[rank]
        assert status == "ok", (rank, info)
        assert info < 1e-4, (rank, info)


@pytest.mark.parametrize("world,E,k,T,chunks", [(2, 8, 2, 37, 2), (4, 16, 4, 37, 3),
                                                 (2, 32, 8, 2, 3)])
def test_ep_chunked_matches_oracle(world, E, k, T, chunks):
    """The pipelined exchange in token chunks (deduplicated rows); with T=2
    rank 0 has fewer tokens than chunks, so one of its chunks is empty while
    rank 1's are not, and both still issue the same collectives."""
    res = run(world, E=E, k=k, T=T, chunks=chunks)
    for rank in range(world):
        status, info = res[rank]
        assert status == "ok", (rank, info)
        assert info < 1e-4, (rank, info)


def test_chunks_need_the_nccl_exchange(tmp_path):
    """chunks > 1 is the NCCL exchange's option and implies dedup."""
    from kernelswift_b200.ep import ExpertParallelMoE

    dist.init_process_group("gloo", store=dist.FileStore(str(tmp_path / "store"), 1),
                            rank=0, world_size=1)
    try:
        w1, w2 = problem(4, 64, 32, seed=1)
        be = CpuBackend(w1, w2)
        with pytest.raises(ValueError, match="chunks"):
            ExpertParallelMoE(None, None, 4, 2, backend=be, exchange="peer", chunks=2)
        with pytest.raises(ValueError, match="chunks"):
            ExpertParallelMoE(None, None, 4, 2, backend=be, chunks=0)
        ep = ExpertParallelMoE(None, None, 4, 2, backend=be, chunks=3)
        assert ep.dedup and ep.chunks == 3 and ep.exchange == "nccl"
    finally:
        dist.destroy_process_group()


def test_dedup_plan_rows():
    """One send row per (token, rank) pair; its ids and weights are exactly the
    token's slots on that rank; inv finds it; counts add up."""
    from kernelswift_b200.ep import dedup_plan

    g = torch.Generator().manual_seed(9)
    T, E, k, world = 53, 32, 8, 4
    w, ids = orc.route(torch.randn(T, E, generator=g) + torch.linspace(0, 2, E), k)
    tokens, eid, sw, inv, counts = dedup_plan(ids, w, E, world)
    el = E // world
    pairs = [(d, t) for d in range(world) for t in range(T)
             if any(int(e) // el == d for e in ids[t])]
    assert tokens.numel() == len(pairs) == int(counts[:world].sum())
    assert int(counts[world]) == 0
    for p, (d, t) in enumerate(pairs):
        assert int(tokens[p]) == t and int(inv[t, d]) == p
        for j in range(k):
            on_d = int(ids[t, j]) // el == d
            assert int(eid[p, j]) == (int(ids[t, j]) - d * el if on_d else -1)
            assert float(sw[p, j]) == (float(w[t, j]) if on_d else 0.0)
    assert int((inv >= 0).sum()) == len(pairs)
    for d in range(world):
        assert int(counts[d]) == sum(1 for dd, _ in pairs if dd == d)


def test_dedup_plan_counts_invalid_ids():
    from kernelswift_b200.ep import dedup_plan

    ids = torch.tensor([[0, 5], [7, 1], [-1, 2]])  # 4 experts on 2 ranks
    w = torch.ones(3, 2)
    tokens, eid, sw, inv, counts = dedup_plan(ids, w, 4, 2)
    # rank 0: tokens 0, 1; rank 1: token 2; all three have an invalid slot
    assert counts.tolist() == [2, 1, 3]
    assert inv.tolist() == [[0, -1], [1, -1], [-1, 2]]
    assert eid.tolist() == [[0, -1], [-1, 1], [-1, 0]]


def test_ep_rank_failure_surfaces_as_error():
    res = run(2, fail_rank=1)
    assert res[1][0] == "error" and "planted failure" in res[1][1]
    # the surviving rank's first collective must fail, not hang
    assert res[0][0] == "error", res[0]


# ---------------------------------------------------------------------------
# The peer-memory exchange's placement rule, restated on gloo ranks: every
# rank learns the full matrix of deduplicated row counts (the kernels write
# rows of it into each other's memory; here all_gather), a sender's rows for
# rank d start at dst_off[d] = sum of what lower ranks send to d, the
# receiver returns one weighted row per (token, rank) over its first n_recv
# rows, and the combine adds, for each token, the rows of the ranks it was
# sent to, read at dst_off[d] + (send row - send_start[d]).
# ---------------------------------------------------------------------------

def peer_worker(rank, world, port, E, k, T, H, I, result_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    try:
        from kernelswift_b200.ep import dedup_plan

        w1, w2 = problem(E, H, I, seed=0)
        el = E // world
        backend = CpuBackend(w1[rank * el:(rank + 1) * el], w2[rank * el:(rank + 1) * el])
        g = torch.Generator().manual_seed(200 + rank)
        Tr = T + 3 * rank  # uneven token counts
        hidden = torch.randn(Tr, H, generator=g)
        logits = torch.randn(Tr, E, generator=g) + torch.linspace(0, 1.5, E)
        w, ids = orc.route(logits, k)
        tokens, send_eid, send_w, inv, counts = dedup_plan(ids, w, E, world)
        # counts matrix on every rank
        mat = [torch.zeros(world, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(mat, counts[:world].clone())
        mat = torch.stack(mat)                        # [s, d]
        send_start = torch.cat([torch.zeros(1, dtype=torch.int64), counts[:world].cumsum(0)])
        dst_off = torch.stack([mat[:rank, d].sum() for d in range(world)])
        n_recv = int(mat[:, rank].sum())
        capacity = (T + 3 * (world - 1)) * world      # max_tokens * world
        # dispatch: rows, ids and weights land at dst_off[d] + i in rank d's buffer
        rows = backend.pack(hidden, tokens, 1)
        recv = torch.zeros(capacity, H)
        recv_id = torch.full((capacity, k), -7, dtype=torch.int32)  # never read past n_recv
        recv_w = torch.zeros(capacity, k)
        for src in range(world):
            part = [torch.zeros(int(mat[src, d]), H) for d in range(world)]
            pid = [torch.zeros(int(mat[src, d]), k, dtype=torch.int32) for d in range(world)]
            pw = [torch.zeros(int(mat[src, d]), k) for d in range(world)]
            if src == rank:
                for d in range(world):
                    sl = slice(int(send_start[d]), int(send_start[d + 1]))
                    part[d], pid[d], pw[d] = rows[sl], send_eid[sl], send_w[sl]
            for d in range(world):
                dist.broadcast(part[d], src)
                dist.broadcast(pid[d], src)
                dist.broadcast(pw[d], src)
            if mat[src, rank] > 0:
                off = int(mat[:src, rank].sum())
                n = int(mat[src, rank])
                recv[off:off + n], recv_id[off:off + n], recv_w[off:off + n] = (
                    part[rank], pid[rank], pw[rank])
        # the expert pass over the first n_recv rows only
        res = torch.zeros(capacity, H)
        res[:n_recv] = backend.experts_weighted(recv[:n_recv], recv_id[:n_recv],
                                                recv_w[:n_recv])
        results = [torch.zeros(capacity, H) for _ in range(world)]
        dist.all_gather(results, res)
        out = torch.zeros(Tr, H)
        for t in range(Tr):
            for d in range(world):
                p = int(inv[t, d])
                if p < 0:
                    continue
                assert int(send_start[d]) <= p < int(send_start[d + 1])
                out[t] += results[d][int(dst_off[d]) + p - int(send_start[d])]
        ref = orc.fused_experts(hidden, w1, w2, w, ids)
        result_q.put((rank, "ok", float((out - ref).abs().max())))
    except Exception as exc:
        result_q.put((rank, "error", repr(exc)[:300]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,E,k", [(2, 8, 2), (4, 16, 4), (4, 32, 8)])
def test_peer_placement_rule_matches_oracle(world, E, k):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=peer_worker, args=(r, world, port, E, k, 21, 64, 32, q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, status, info in res:
        assert status == "ok", (rank, info)
        assert info < 1e-4, (rank, info)
