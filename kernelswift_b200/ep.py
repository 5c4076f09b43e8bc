"""Expert parallelism for the fused-MoE operator (one process per GPU).

Experts are sharded in contiguous blocks: with E experts over `world` ranks,
rank r holds experts [r*E/world, (r+1)*E/world). Tokens stay data-parallel:
every rank routes its own tokens. One forward is

  1. plan (moe_ep_plan, one launch): dest[r] = topk_ids[r] // E_local for
     every flat slot r = t*k + j; `order` = the slots sorted by destination
     rank (stable), the destination-local expert ids in that order, the
     inverse permutation and the per-destination counts
  2. all_to_all of the per-destination counts (the only host sync: NCCL's
     variable-size all_to_all needs the split sizes on the host)
  3. pack: send_rows[i] = hidden[order[i] // k]       (moe_gather_rows)
  4. all_to_all of the packed rows and of their destination-local expert ids
  5. local experts on the received rows: moe_fused_experts with top_k = 1
     and unit weights (the topk weight is applied on the way back)
  6. all_to_all of the result rows back to their source ranks
  7. combine: out[t] = sum_j w[t,j] * rows[inv[t*k+j]]  (moe_combine_rows)

This replaces, across ranks, the expert loop and weighted sum of
kernels/track1-triton/fused_moe/base.py:64-76. The collectives run over
torch.distributed (NCCL over NVLink/NVSwitch on B200); every rank issues the
same collectives in the same order, so a rank that fails makes the others'
next collective end with the process group's timeout instead of hanging.

The device work (plan, pack, local experts, combine) goes through a backend
object;
`CudaBackend` runs the library's kernels and is the only backend this package
provides.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib
from . import fused_moe as fm


class CudaBackend:
    """Device work of an EP forward on the libmoe_b200 kernels."""

    def __init__(self, prepared: fm.PreparedWeights, quant: str = "none"):
        self.prep = prepared
        self.quant = quant

    def plan(self, topk_ids: torch.Tensor, num_experts: int, world: int):
        """(order, send_eid, inv, counts) of moe_ep_plan for this rank's ids."""
        ids = topk_ids.reshape(-1).contiguous()
        n = ids.numel()
        dev = ids.device
        order = torch.empty(n, dtype=torch.int32, device=dev)
        send_eid = torch.empty(n, dtype=torch.int32, device=dev)
        inv = torch.empty(n, dtype=torch.int32, device=dev)
        counts = torch.empty(world + 1, dtype=torch.int64, device=dev)
        _lib.call("moe_ep_plan", fm._ptr(ids), fm._code(ids), n, num_experts, world,
                  fm._ptr(order), fm._ptr(send_eid), fm._ptr(inv), fm._ptr(counts),
                  fm._stream(dev))
        return order, send_eid, inv, counts

    def pack(self, hidden: torch.Tensor, order: torch.Tensor, top_k: int) -> torch.Tensor:
        n = order.numel()
        rows = torch.empty(n, hidden.shape[1], dtype=hidden.dtype, device=hidden.device)
        if n == 0:
            return rows
        order32 = order.to(torch.int32)
        count = torch.full((1,), n, dtype=torch.int32, device=hidden.device)
        code = fm._code(hidden)
        _lib.call("moe_gather_rows", fm._ptr(hidden), code, hidden.shape[0], hidden.shape[1],
                  top_k, fm._ptr(order32), fm._ptr(count), n, n, _lib.QUANT_NONE,
                  fm._ptr(rows), code, None, fm._stream(hidden.device))
        return rows

    def experts(self, rows: torch.Tensor, local_ids: torch.Tensor,
                stage_events=None) -> torch.Tensor:
        ones = torch.ones(rows.shape[0], 1, dtype=torch.float32, device=rows.device)
        return fm.fused_experts(rows, self.prep, None, ones, local_ids.view(-1, 1),
                                use_fp8_w8a8=self.quant == "fp8",
                                use_int8_w8a8=self.quant == "int8", stage_events=stage_events)

    def combine(self, rows: torch.Tensor, inv: torch.Tensor, weights: torch.Tensor,
                num_tokens: int, top_k: int) -> torch.Tensor:
        H = rows.shape[1]
        out = torch.empty(num_tokens, H, dtype=rows.dtype, device=rows.device)
        if num_tokens == 0:
            return out
        w = weights.reshape(-1).contiguous()
        inv32 = inv.to(torch.int32).contiguous()
        _lib.call("moe_combine_rows", fm._ptr(rows), fm._code(rows), fm._ptr(inv32), fm._ptr(w),
                  fm._code(w), num_tokens, top_k, H, fm._ptr(out), fm._code(out),
                  fm._stream(rows.device))
        return out


class ExpertParallelMoE:
    """Fused MoE with experts sharded over the ranks of `group`.

    w1_local [E_local, 2I, H] and w2_local [E_local, H, I] are this rank's
    experts (global ids rank*E_local ...); `forward(hidden, topk_weights,
    topk_ids)` takes this rank's tokens with GLOBAL expert ids and returns
    their outputs [T, H].
    """

    def __init__(self, w1_local: torch.Tensor | None, w2_local: torch.Tensor | None,
                 num_experts: int, top_k: int, group=None, quant: str = "none",
                 backend=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if num_experts % self.world:
            raise ValueError(f"{num_experts} experts do not shard over {self.world} ranks")
        self.num_experts = num_experts
        self.e_local = num_experts // self.world
        self.top_k = top_k
        if backend is None:
            if w1_local is None or w1_local.shape[0] != self.e_local:
                raise ValueError(f"this rank needs w1 for {self.e_local} experts")
            compute = torch.bfloat16 if w1_local.dtype != torch.float16 else torch.float16
            backend = CudaBackend(fm.prepare_weights(w1_local, w2_local, quant, compute), quant)
        self.backend = backend

    def forward(self, hidden: torch.Tensor, topk_weights: torch.Tensor,
                topk_ids: torch.Tensor, stage_events=None) -> torch.Tensor:
        """`stage_events` (fused_moe.stage_event_array) times the launches of
        the local expert computation."""
        T, H = hidden.shape
        k = topk_ids.shape[1]
        dev = hidden.device
        numel = topk_ids.numel()
        order, send_eid, inv, counts = self.backend.plan(topk_ids, self.num_experts, self.world)
        recv_counts = torch.empty(self.world, dtype=counts.dtype, device=dev)
        dist.all_to_all_single(recv_counts, counts[:self.world].contiguous(), group=self.group)
        both = torch.cat([counts, recv_counts]).cpu()  # the one host sync
        send_split = both[:self.world].tolist()
        recv_split = both[self.world + 1:].tolist()
        n_recv = sum(recv_split)
        if int(both[self.world]) != 0:
            raise ValueError("expert ids out of range")
        n_send = numel
        order = order[:n_send]
        send_eid = send_eid[:n_send]

        send_rows = self.backend.pack(hidden, order, k)
        recv_rows = torch.empty(n_recv, H, dtype=hidden.dtype, device=dev)
        recv_eid = torch.empty(n_recv, dtype=torch.int32, device=dev)
        dist.all_to_all_single(recv_rows, send_rows, recv_split, send_split, group=self.group)
        dist.all_to_all_single(recv_eid, send_eid, recv_split, send_split, group=self.group)

        self.last_rows_received = n_recv
        if stage_events is not None:
            out_rows = self.backend.experts(recv_rows, recv_eid, stage_events=stage_events)
        else:
            out_rows = self.backend.experts(recv_rows, recv_eid)
        back = torch.empty(n_send, H, dtype=out_rows.dtype, device=dev)
        dist.all_to_all_single(back, out_rows, send_split, recv_split, group=self.group)
        return self.backend.combine(back, inv, topk_weights, T, k)

    __call__ = forward
