"""Expert parallelism for the fused-MoE operator (one process per GPU).

Experts are sharded in contiguous blocks: with E experts over `world` ranks,
rank r holds experts [r*E/world, (r+1)*E/world). Tokens stay data-parallel:
every rank routes its own tokens. One forward is

  1. plan (moe_ep_plan_ws: one launch up to 8192 slots, three above):
     dest[r] = topk_ids[r] // E_local for every flat slot r = t*k + j;
     `order` = the slots sorted by destination
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

Deduplicated exchange: a token is sent to a rank once, however many of its
k slots that rank holds (top-8 of 256 experts over 8 ranks reaches about 5.3
ranks per token, so a third of the rows stay home). The plan is one kernel
(moe_ep_plan_dedup; `dedup_plan` restates it in torch for CPU backends): the
send row carries the token's expert ids local to that rank (-1 for slots
elsewhere) and their weights, the receiver runs moe_fused_experts with top_k
= k (slots marked -1 are dropped) and returns one weighted, summed row per
(token, rank), and the source adds the rows of the ranks it used. The NCCL
exchange does this with dedup=True; the peer exchange always does.

Chunked NCCL exchange (chunks=C > 1, deduplicated rows): the tokens are cut
into C contiguous chunks, planned up front (C plan launches, one all_to_all
of the [world, C] count matrix, one host sync), and pipelined: chunk c+1's
rows, ids and weights are sent (async all_to_all) before chunk c's experts
are enqueued, and chunk c's result rows return (async) while chunk c+1's
experts run. ProcessGroupNCCL runs the collectives on its own stream, which
waits for the work enqueued before each collective, so the transfer of one
chunk overlaps the expert GEMMs of the previous one. Every rank cuts its own
tokens into the same number of chunks (a chunk may be empty), so all ranks
issue the same collectives in the same order.

With exchange="peer" (ranks on one node, 2-8 GPUs) the all_to_alls are
replaced by two kernels that move the rows themselves over NVLink
(`PeerExchange`, the moe_ep_peer_* entry points): dispatch stores each
deduplicated row with its ids and weights into the destination GPU's
receive buffer (mapped with CUDA IPC) at an offset every rank derives from a
counts matrix the ranks write into each other's memory, and combine loads
each rank's result row from the GPU that computed it. The ranks hand off
through flags in each other's memory, so a step needs no host
synchronisation and no NCCL call. The receive buffer is sized for the worst
case (max_tokens * world rows); the local expert pass reads the count the
dispatch stored on the device (num_tokens_dev) and touches only the rows
that arrived.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib
from . import fused_moe as fm


def dedup_plan(topk_ids: torch.Tensor, topk_weights: torch.Tensor, num_experts: int,
               world: int):
    """Send plan with one row per (token, destination rank) holding any of
    the token's slots (dedup=True). Returns

      tokens   int32 [n]      source token of send row p, rows grouped by
                              destination rank (ascending), tokens ascending
                              inside a rank
      send_eid int32 [n, k]   the token's expert ids local to that rank, -1 for
                              slots held elsewhere
      send_w   f32   [n, k]   their weights (0 for slots held elsewhere)
      inv      int32 [T, world] send row of (token, rank), -1 if none
      counts   int64 [world + 1] rows per rank; counts[world] = tokens with an
                              expert id outside [0, num_experts)

    Plain torch ops, so the same code runs on the GPU and in CPU tests."""
    T, k = topk_ids.shape
    dev = topk_ids.device
    el = num_experts // world
    ids = topk_ids.long()
    valid = (ids >= 0) & (ids < num_experts)
    dest = torch.where(valid, torch.div(ids, el, rounding_mode="floor"),
                       torch.full_like(ids, world))
    present = torch.zeros(world + 1, T, dtype=torch.bool, device=dev)
    present.scatter_(0, dest.t().contiguous(), True)
    counts = present.sum(1)
    d_idx, t_idx = present[:world].nonzero(as_tuple=True)
    sel = dest[t_idx] == d_idx.unsqueeze(1)
    send_eid = torch.where(sel, ids[t_idx] - d_idx.unsqueeze(1) * el,
                           torch.full_like(ids[t_idx], -1)).to(torch.int32)
    send_w = torch.where(sel, topk_weights[t_idx].float(),
                         torch.zeros(sel.shape, dtype=torch.float32, device=dev))
    inv = torch.full((T, world), -1, dtype=torch.int32, device=dev)
    inv[t_idx, d_idx] = torch.arange(t_idx.numel(), dtype=torch.int32, device=dev)
    return t_idx.to(torch.int32), send_eid, send_w, inv, counts


class CudaBackend:
    """Device work of an EP forward on the libmoe_b200 kernels."""

    def __init__(self, prepared: fm.PreparedWeights, quant: str = "none"):
        self.prep = prepared
        self.quant = quant
        self._plan_ws = None

    def plan(self, topk_ids: torch.Tensor, num_experts: int, world: int):
        """(order, send_eid, inv, counts) of moe_ep_plan for this rank's ids
        (moe_ep_plan_ws: more than 8192 slots are spread over CTAs)."""
        ids = topk_ids.reshape(-1).contiguous()
        n = ids.numel()
        dev = ids.device
        order = torch.empty(n, dtype=torch.int32, device=dev)
        send_eid = torch.empty(n, dtype=torch.int32, device=dev)
        inv = torch.empty(n, dtype=torch.int32, device=dev)
        counts = torch.empty(world + 1, dtype=torch.int64, device=dev)
        nbytes = ctypes.c_size_t(0)
        _lib.call("moe_ep_plan_workspace_size", n, world, ctypes.byref(nbytes))
        if self._plan_ws is None or self._plan_ws.numel() < nbytes.value:
            self._plan_ws = torch.empty(max(nbytes.value, 256), dtype=torch.uint8, device=dev)
        _lib.call("moe_ep_plan_ws", fm._ptr(ids), fm._code(ids), n, num_experts, world,
                  fm._ptr(order), fm._ptr(send_eid), fm._ptr(inv), fm._ptr(counts),
                  fm._ptr(self._plan_ws), self._plan_ws.numel(), fm._stream(dev))
        return order, send_eid, inv, counts

    def plan_dedup(self, topk_ids: torch.Tensor, topk_weights: torch.Tensor, num_experts: int,
                   world: int):
        """dedup_plan's outputs from one kernel (moe_ep_plan_dedup); row
        buffers are sized for num_tokens * world rows, counts[:world] says
        how many are used."""
        T, k = topk_ids.shape
        dev = topk_ids.device
        ids = topk_ids.contiguous()
        w = topk_weights.contiguous()
        n = T * world
        tokens = torch.empty(n, dtype=torch.int32, device=dev)
        send_eid = torch.empty(n, k, dtype=torch.int32, device=dev)
        send_w = torch.empty(n, k, dtype=torch.float32, device=dev)
        inv = torch.empty(T, world, dtype=torch.int32, device=dev)
        counts = torch.empty(world + 1, dtype=torch.int64, device=dev)
        _lib.call("moe_ep_plan_dedup", fm._ptr(ids), fm._code(ids), fm._ptr(w), fm._code(w), T,
                  k, num_experts, world, fm._ptr(tokens), fm._ptr(send_eid), fm._ptr(send_w),
                  fm._ptr(inv), fm._ptr(counts), fm._stream(dev))
        return tokens, send_eid, send_w, inv, counts

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
                                use_fp8_w8a8=self.quant.startswith("fp8"),
                                use_int8_w8a8=self.quant == "int8", stage_events=stage_events)

    def experts_weighted(self, rows: torch.Tensor, local_ids: torch.Tensor,
                         weights: torch.Tensor, stage_events=None) -> torch.Tensor:
        """sum_j weights[:, j] * expert_{local_ids[:, j]}(rows) (ids -1 dropped)."""
        return fm.fused_experts(rows, self.prep, None, weights, local_ids,
                                use_fp8_w8a8=self.quant.startswith("fp8"),
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


class _DeviceArray:
    """__cuda_array_interface__ of device memory the library owns."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                         "data": (int(ptr), False), "version": 3,
                                         "strides": None}


class PeerExchange:
    """This rank's moe_ep_peer buffer, connected to every rank's buffer.

    Collective: every rank of `group` constructs it with the same capacity,
    hidden size and dtype (the IPC handles are exchanged with
    all_gather_object). `close()` is collective too.
    """

    def __init__(self, group, world: int, rank: int, capacity: int, hidden_size: int,
                 top_k: int, dtype: torch.dtype, device: torch.device, wait_limit_ms: int = 0):
        if dtype not in (torch.bfloat16, torch.float16):
            raise ValueError("the peer exchange moves f16/bf16 rows")
        self.group = group
        self.device = device
        self.capacity = capacity
        self.dtype = dtype
        self.handle = None
        handle = ctypes.c_void_p()
        raw = (ctypes.c_uint8 * _lib.EP_HANDLE_BYTES)()
        lib = _lib.load()
        # every step below is agreed on by all ranks, so that a failure on one
        # rank raises on all of them instead of leaving the others in a
        # collective
        st = lib.moe_ep_peer_create(world, rank, capacity, hidden_size, top_k,
                                    fm._code(torch.empty(0, dtype=dtype)), wait_limit_ms,
                                    ctypes.byref(handle), raw)
        detail = lib.moe_last_error().decode() if st else ""
        if not self._all_ok(st == 0):
            if st == 0:
                lib.moe_ep_peer_destroy(handle)
            raise RuntimeError(f"peer exchange unavailable (rank {rank}: {detail or 'ok'})")
        handles = [None] * world
        dist.all_gather_object(handles, bytes(raw), group=group)
        st = lib.moe_ep_peer_connect(handle, b"".join(handles))
        detail = lib.moe_last_error().decode() if st else ""
        if not self._all_ok(st == 0):
            lib.moe_ep_peer_disconnect(handle)
            dist.barrier(group=group)
            lib.moe_ep_peer_destroy(handle)
            raise RuntimeError(f"peer exchange unavailable (rank {rank}: {detail or 'ok'})")
        self.handle = handle
        rows, ids, wts, res, cnt = (ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_void_p(),
                                    ctypes.c_void_p(), ctypes.c_void_p())
        _lib.call("moe_ep_peer_buffers", handle, ctypes.byref(rows), ctypes.byref(ids),
                  ctypes.byref(wts), ctypes.byref(res), ctypes.byref(cnt))
        shape = (capacity, hidden_size)
        self.top_k = top_k
        self.recv_rows = torch.as_tensor(_DeviceArray(rows.value, shape, "<i2"),
                                         device=device).view(dtype)
        self.recv_ids = torch.as_tensor(_DeviceArray(ids.value, (capacity, top_k), "<i4"),
                                        device=device)
        self.recv_weights = torch.as_tensor(_DeviceArray(wts.value, (capacity, top_k), "<f4"),
                                            device=device)
        self.result_rows = torch.as_tensor(_DeviceArray(res.value, shape, "<i2"),
                                           device=device).view(dtype)
        # rows the last dispatch delivered (written by the dispatch kernel)
        self.recv_count = torch.as_tensor(_DeviceArray(cnt.value, (1,), "<i4"), device=device)
        self.status = torch.zeros(1, dtype=torch.int32, device=device)

    def _all_ok(self, ok: bool) -> bool:
        """True when `ok` holds on every rank of the group (collective)."""
        on_gpu = dist.get_backend(self.group) == "nccl"
        t = torch.tensor([1 if ok else 0], dtype=torch.int32,
                         device=self.device if on_gpu else "cpu")
        dist.all_reduce(t, op=dist.ReduceOp.MIN, group=self.group)
        return bool(t.item())

    def all_ok(self) -> bool:
        """Collective: True when no rank's exchange kernels recorded an error."""
        return self._all_ok(int(self.status.item()) == 0)

    def check(self) -> None:
        """Raises if a kernel of the exchange recorded an error (synchronises)."""
        code = int(self.status.item())
        if code:
            raise _lib.MoeError(code, "expert-parallel peer exchange",
                                "a rank did not arrive in time or a receive buffer overflowed")

    def close(self) -> None:
        """Collective: unmaps the other ranks' buffers, then frees this one."""
        if self.handle is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        _lib.load().moe_ep_peer_disconnect(self.handle)
        dist.barrier(group=self.group)
        self.recv_rows = self.recv_ids = self.recv_weights = self.result_rows = None
        self.recv_count = None
        _lib.call("moe_ep_peer_destroy", self.handle)
        self.handle = None


# the stages of an expert-parallel step that `exchange_events` brackets
EXCHANGE_STAGES = ("plan", "dispatch", "experts", "combine")


class ExpertParallelMoE:
    """Fused MoE with experts sharded over the ranks of `group`.

    w1_local [E_local, 2I, H] and w2_local [E_local, H, I] are this rank's
    experts (global ids rank*E_local ...); `forward(hidden, topk_weights,
    topk_ids)` takes this rank's tokens with GLOBAL expert ids and returns
    their outputs [T, H].
    """

    def __init__(self, w1_local: torch.Tensor | None, w2_local: torch.Tensor | None,
                 num_experts: int, top_k: int, group=None, quant: str = "none",
                 backend=None, exchange: str = "auto", max_tokens: int | None = None,
                 dtype: torch.dtype = torch.bfloat16, wait_limit_ms: int = 0,
                 dedup: bool = False, chunks: int = 1):
        """exchange: "nccl" (all_to_all), "peer" (NVLink peer memory, needs
        max_tokens: the most tokens a rank passes to one forward) or "auto"
        (peer when max_tokens is given, the CUDA backend is used and the
        group has 2-8 ranks on GPUs, else nccl). `dtype` is the row dtype of
        the peer exchange (the hidden states' dtype). dedup: send a token to
        a rank once however many of its slots the rank holds (the NCCL
        exchange's option; the peer exchange always does). chunks > 1: the
        NCCL exchange in that many token chunks, each chunk's transfer
        overlapping the previous chunk's experts (implies dedup; not for the
        peer exchange)."""
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
        self.quant = quant
        if exchange == "auto":
            exchange = ("peer" if max_tokens is not None and isinstance(backend, CudaBackend)
                        and 2 <= self.world <= _lib.EP_MAX_RANKS else "nccl")
        if exchange not in ("nccl", "peer"):
            raise ValueError(f"unknown exchange {exchange!r}")
        if chunks < 1 or (chunks > 1 and exchange != "nccl"):
            raise ValueError("chunks must be >= 1, and > 1 only with the NCCL exchange")
        self.exchange = exchange
        self.chunks = chunks
        self.dedup = dedup or exchange == "peer" or chunks > 1
        self._last_recv_eid = None
        self._evs = None
        self.peer = None
        self.max_tokens = max_tokens
        self.last_rows_received = 0
        if exchange == "peer":
            if max_tokens is None or not isinstance(backend, CudaBackend):
                raise ValueError("the peer exchange needs max_tokens and the CUDA backend")
            dev = backend.prep.w13.device
            # worst case: every token of every rank has a slot on this rank
            self.peer = PeerExchange(group, self.world, self.rank, max_tokens * self.world,
                                     backend.prep.hidden_size, top_k, dtype, dev, wait_limit_ms)

    def forward(self, hidden: torch.Tensor, topk_weights: torch.Tensor,
                topk_ids: torch.Tensor, stage_events=None, exchange_events=None) -> torch.Tensor:
        """`stage_events` (fused_moe.stage_event_array) times the launches of
        the local expert computation. `exchange_events`, a list of
        len(EXCHANGE_STAGES) + 1 torch.cuda.Event, is recorded on the current
        stream at the boundaries of the step's exchange stages (plan,
        dispatch, local experts, combine)."""
        self._evs = exchange_events
        if self.peer is not None:
            return self._forward_peer(hidden, topk_weights, topk_ids, stage_events)
        if self.chunks > 1:
            return self._forward_chunked(hidden, topk_weights, topk_ids, stage_events)
        if self.dedup:
            return self._forward_dedup(hidden, topk_weights, topk_ids, stage_events)
        T, H = hidden.shape
        k = topk_ids.shape[1]
        dev = hidden.device
        numel = topk_ids.numel()
        self._mark(0)
        order, send_eid, inv, counts = self.backend.plan(topk_ids, self.num_experts, self.world)
        self._mark(1)
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
        self._mark(2)
        if stage_events is not None:
            out_rows = self.backend.experts(recv_rows, recv_eid, stage_events=stage_events)
        else:
            out_rows = self.backend.experts(recv_rows, recv_eid)
        self._mark(3)
        back = torch.empty(n_send, H, dtype=out_rows.dtype, device=dev)
        dist.all_to_all_single(back, out_rows, send_split, recv_split, group=self.group)
        out = self.backend.combine(back, inv, topk_weights, T, k)
        self._mark(4)
        return out

    def _forward_dedup(self, hidden, topk_weights, topk_ids, stage_events=None):
        T, H = hidden.shape
        k = topk_ids.shape[1]
        dev = hidden.device
        self._mark(0)
        if hasattr(self.backend, "plan_dedup"):
            tokens, send_eid, send_w, inv, counts = self.backend.plan_dedup(
                topk_ids, topk_weights, self.num_experts, self.world)
        else:
            tokens, send_eid, send_w, inv, counts = dedup_plan(topk_ids, topk_weights,
                                                               self.num_experts, self.world)
        self._mark(1)
        recv_counts = torch.empty(self.world, dtype=counts.dtype, device=dev)
        dist.all_to_all_single(recv_counts, counts[:self.world].contiguous(), group=self.group)
        both = torch.cat([counts, recv_counts]).cpu()  # the one host sync
        if int(both[self.world]) != 0:
            raise ValueError("expert ids out of range")
        send_split = both[:self.world].tolist()
        recv_split = both[self.world + 1:].tolist()
        n_recv = sum(recv_split)
        n_send = sum(send_split)
        tokens, send_eid, send_w = tokens[:n_send], send_eid[:n_send], send_w[:n_send]
        send_rows = self.backend.pack(hidden, tokens, 1)
        recv_rows = torch.empty(n_recv, H, dtype=hidden.dtype, device=dev)
        recv_eid = torch.empty(n_recv, k, dtype=torch.int32, device=dev)
        recv_w = torch.empty(n_recv, k, dtype=torch.float32, device=dev)
        dist.all_to_all_single(recv_rows, send_rows, recv_split, send_split, group=self.group)
        dist.all_to_all_single(recv_eid, send_eid, recv_split, send_split, group=self.group)
        dist.all_to_all_single(recv_w, send_w, recv_split, send_split, group=self.group)
        self.last_rows_received = n_recv
        self._last_recv_eid = recv_eid
        self._mark(2)
        if stage_events is not None:
            out_rows = self.backend.experts_weighted(recv_rows, recv_eid, recv_w,
                                                     stage_events=stage_events)
        else:
            out_rows = self.backend.experts_weighted(recv_rows, recv_eid, recv_w)
        self._mark(3)
        back = torch.empty(tokens.numel(), H, dtype=out_rows.dtype, device=dev)
        dist.all_to_all_single(back, out_rows, send_split, recv_split, group=self.group)
        ones = torch.ones(T, self.world, dtype=torch.float32, device=dev)
        out = self.backend.combine(back, inv.reshape(-1), ones, T, self.world)
        self._mark(4)
        return out

    def _plan_dedup(self, topk_ids, topk_weights):
        if hasattr(self.backend, "plan_dedup"):
            return self.backend.plan_dedup(topk_ids, topk_weights, self.num_experts, self.world)
        return dedup_plan(topk_ids, topk_weights, self.num_experts, self.world)

    def _forward_chunked(self, hidden, topk_weights, topk_ids, stage_events=None):
        """The deduplicated NCCL exchange in self.chunks pipelined token chunks
        (module docstring). Exchange events: 0 before the plans, 1 after them,
        2 when chunk 0's rows have arrived, 3 after the last chunk's experts,
        4 after the last combine."""
        T, H = hidden.shape
        k = topk_ids.shape[1]
        dev = hidden.device
        world, C = self.world, self.chunks
        bounds = [T * c // C for c in range(C + 1)]
        self._mark(0)
        plans = [self._plan_dedup(topk_ids[bounds[c]:bounds[c + 1]],
                                  topk_weights[bounds[c]:bounds[c + 1]]) for c in range(C)]
        self._mark(1)
        counts = torch.stack([p[4][:world + 1] for p in plans])  # [C, world + 1]
        send_counts = counts[:, :world].t().contiguous()  # [world, C]: per destination
        recv_counts = torch.empty_like(send_counts)
        dist.all_to_all_single(recv_counts, send_counts, group=self.group)
        both = torch.cat([counts.reshape(-1), recv_counts.reshape(-1)]).cpu()  # one host sync
        cnt = both[:C * (world + 1)].view(C, world + 1)
        rcv = both[C * (world + 1):].view(world, C)
        if int(cnt[:, world].sum()) != 0:
            raise ValueError("expert ids out of range")

        def dispatch(c):
            tokens, send_eid, send_w, inv, _ = plans[c]
            send_split = cnt[c, :world].tolist()
            recv_split = rcv[:, c].tolist()
            n_send, n_recv = sum(send_split), sum(recv_split)
            rows = self.backend.pack(hidden[bounds[c]:bounds[c + 1]], tokens[:n_send], 1)
            recv_rows = torch.empty(n_recv, H, dtype=hidden.dtype, device=dev)
            recv_eid = torch.empty(n_recv, k, dtype=torch.int32, device=dev)
            recv_w = torch.empty(n_recv, k, dtype=torch.float32, device=dev)
            works = [dist.all_to_all_single(recv_rows, rows, recv_split, send_split,
                                            group=self.group, async_op=True),
                     dist.all_to_all_single(recv_eid, send_eid[:n_send], recv_split, send_split,
                                            group=self.group, async_op=True),
                     dist.all_to_all_single(recv_w, send_w[:n_send], recv_split, send_split,
                                            group=self.group, async_op=True)]
            # the send buffers stay referenced until the collectives are waited on
            return {"c": c, "send_split": send_split, "recv_split": recv_split, "inv": inv,
                    "rows": recv_rows, "eid": recv_eid, "w": recv_w, "works": works,
                    "n_send": n_send, "sent": (rows, send_eid, send_w)}

        out = torch.empty(T, H, dtype=hidden.dtype, device=dev)
        returning = []
        received = []
        nxt = dispatch(0)
        for c in range(C):
            cur = nxt
            for w in cur["works"]:
                w.wait()
            if c == 0:
                self._mark(2)
            if c + 1 < C:
                nxt = dispatch(c + 1)  # in flight during this chunk's experts
            received.append(cur["eid"])
            if stage_events is not None and c == 0:
                rows = self.backend.experts_weighted(cur["rows"], cur["eid"], cur["w"],
                                                     stage_events=stage_events)
            else:
                rows = self.backend.experts_weighted(cur["rows"], cur["eid"], cur["w"])
            back = torch.empty(cur["n_send"], H, dtype=rows.dtype, device=dev)
            work = dist.all_to_all_single(back, rows, cur["send_split"], cur["recv_split"],
                                          group=self.group, async_op=True)
            returning.append((cur, back, work, rows))
        self._mark(3)
        for cur, back, work, _rows in returning:
            work.wait()
            c = cur["c"]
            t_c = bounds[c + 1] - bounds[c]
            if t_c == 0:
                continue
            ones = torch.ones(t_c, world, dtype=torch.float32, device=dev)
            out[bounds[c]:bounds[c + 1]] = self.backend.combine(back, cur["inv"].reshape(-1),
                                                                ones, t_c, world)
        self._mark(4)
        self._last_recv_eid = torch.cat(received)
        self.last_rows_received = sum(int(e.shape[0]) for e in received)
        return out

    def _forward_peer(self, hidden, topk_weights, topk_ids, stage_events=None):
        px = self.peer
        T, H = hidden.shape
        k = topk_ids.shape[1]
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens exceed max_tokens={self.max_tokens}")
        if hidden.dtype != px.dtype:
            raise ValueError(f"hidden states are {hidden.dtype}, the exchange moves {px.dtype}")
        if k != px.top_k:
            raise ValueError(f"top_k {k} differs from the exchange's {px.top_k}")
        dev = hidden.device
        stream = fm._stream(dev)
        # a misaligned view is copied: no rank's dispatch is refused while its peers wait
        hidden = fm._contig(hidden)
        self._mark(0)
        tokens, send_eid, send_w, inv, counts = self.backend.plan_dedup(
            topk_ids, topk_weights, self.num_experts, self.world)
        self._mark(1)
        _lib.call("moe_ep_peer_dispatch", px.handle, fm._ptr(hidden), T, fm._ptr(tokens),
                  fm._ptr(send_eid), fm._ptr(send_w), fm._ptr(counts), fm._ptr(px.status),
                  stream)
        self._mark(2)
        # the received rows: one per (token, this rank), k local ids and
        # weights each; only the first recv_count rows (on the device) exist
        fm.fused_experts(px.recv_rows, self.backend.prep, None, px.recv_weights, px.recv_ids,
                         use_fp8_w8a8=self.quant.startswith("fp8"),
                         use_int8_w8a8=self.quant == "int8", out=px.result_rows,
                         status=px.status, stage_events=stage_events,
                         num_tokens_dev=px.recv_count)
        self._mark(3)
        out = torch.empty(T, H, dtype=hidden.dtype, device=dev)
        _lib.call("moe_ep_peer_combine", px.handle, fm._ptr(inv), T, fm._ptr(out),
                  fm._ptr(px.status), stream)
        self._mark(4)
        return out

    def _mark(self, i: int) -> None:
        """Records exchange event i of this step, if the caller passed some."""
        if self._evs is not None:
            self._evs[i].record()

    def rows_received(self) -> int:
        """Rows this rank's experts processed in the last forward, i.e. routed
        (token, slot) pairs (synchronises in the peer and dedup exchanges;
        `last_rows_received` counts the token rows that crossed)."""
        if self.peer is not None:
            n = int(self.peer.recv_count.item())
            return int((self.peer.recv_ids[:n] >= 0).sum())
        if self.dedup:
            return int((self._last_recv_eid >= 0).sum())
        return self.last_rows_received

    def close(self) -> None:
        """Collective: releases the peer exchange buffers (no-op for nccl)."""
        if self.peer is not None:
            self.peer.close()
            self.peer = None

    __call__ = forward
