"""Fused-MoE operator for B200: the host side above the C ABI.

Mirrors the reference operator kernels/track1-triton/fused_moe/base.py:
  - `ModelNew(num_experts, top_k, hidden_size, intermediate_size, renormalize)`
    with parameters `w1` [E, 2I, H] and `w2` [E, H, I] (base.py:9-33) and
    `forward(hidden_states, router_logits)` (base.py:35-76), so that
    auto_bench.py's v0/v1 comparison loads it unchanged;
  - the functional pieces of that forward: `fused_topk` (routing,
    base.py:44-48), `moe_align_block_size` (the per-expert grouping of
    base.py:64-68) and `fused_experts` (base.py:50-76), which also accepts
    fp8 block-scaled and int8 per-channel W8A8 weights.

Device memory, streams and routing ops come from PyTorch; every expert
computation runs in libmoe_b200.so (sm_100a). There is no CPU fallback:
CPU tensors or a missing library raise.
"""
from __future__ import annotations

import ctypes
import threading
import weakref
from dataclasses import dataclass

import torch
import torch.nn as nn

from . import _lib

BLOCK_M = 128

_DTYPE_CODE = {
    torch.float32: _lib.DT_F32,
    torch.float16: _lib.DT_F16,
    torch.bfloat16: _lib.DT_BF16,
    torch.float8_e4m3fn: _lib.DT_E4M3,
    torch.int8: _lib.DT_I8,
    torch.int32: _lib.DT_I32,
    torch.int64: _lib.DT_I64,
}

_QUANT = {"none": _lib.QUANT_NONE, "fp8": _lib.QUANT_FP8_BLOCK, "int8": _lib.QUANT_INT8_CHANNEL,
          "fp8-ue8m0": _lib.QUANT_FP8_UE8M0}


def _code(t: torch.Tensor) -> int:
    try:
        return _DTYPE_CODE[t.dtype]
    except KeyError:
        raise TypeError(f"unsupported dtype {t.dtype}") from None


def _ptr(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(device: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _check_cuda(name: str, t: torch.Tensor) -> None:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (this operator has no CPU path)")


def _contig(t: torch.Tensor) -> torch.Tensor:
    """A dense tensor whose data starts on a 16-byte boundary (the kernels
    move rows in 16-byte vectors): `t` itself when it already is one, else a
    copy (a view that starts mid-row of a larger tensor, for instance)."""
    if t.is_contiguous() and t.data_ptr() % 16 == 0:
        return t
    return t.clone(memory_format=torch.contiguous_format)


# ---------------------------------------------------------------------------
# Workspace: one grow-only buffer per (device, stream) so that calls never
# allocate once warm.
# ---------------------------------------------------------------------------
_ws_lock = threading.Lock()
_ws: dict[tuple[int, int], torch.Tensor] = {}
# buffers replaced after a CUDA graph captured them: a graph keeps using the
# addresses it recorded, so these stay allocated for the life of the process
_ws_captured: list[torch.Tensor] = []
_ws_in_graph: set[int] = set()


def _workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    key = (device.index if device.index is not None else torch.cuda.current_device(),
           torch.cuda.current_stream(device).cuda_stream)
    capturing = torch.cuda.is_current_stream_capturing()
    with _ws_lock:
        buf = _ws.get(key)
        if buf is None or buf.numel() < nbytes:
            if buf is not None and buf.data_ptr() in _ws_in_graph:
                _ws_captured.append(buf)
            buf = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=device)
            _ws[key] = buf
        if capturing:
            _ws_in_graph.add(buf.data_ptr())
        return buf


# ---------------------------------------------------------------------------
# Routing (base.py:44-48)
# ---------------------------------------------------------------------------

def fused_topk(hidden_states: torch.Tensor, gating_output: torch.Tensor, topk: int,
               renormalize: bool = True, weights_dtype: torch.dtype = torch.float32,
               ids_dtype: torch.dtype = torch.int32) -> tuple[torch.Tensor, torch.Tensor]:
    """softmax(fp32) -> top-k -> optional renormalisation, in one kernel.

    The routing of base.py:44-48 (moe_topk_softmax): experts are selected by
    logit, largest first, ties to the lower index; the weights are the fp32
    softmax probabilities of the selected experts, renormalised to sum to 1
    when `renormalize`, returned in `weights_dtype` (base.py:48 casts them to
    the activation dtype). Returns (topk_weights [T, k], topk_ids [T, k]).
    """
    _check_cuda("gating_output", gating_output)
    if gating_output.dim() != 2 or gating_output.shape[0] != hidden_states.shape[0]:
        raise ValueError("gating_output must be [T, E] with T = hidden_states.shape[0]")
    logits = _contig(gating_output)
    T, E = logits.shape
    dev = logits.device
    w = torch.empty(T, topk, dtype=weights_dtype, device=dev)
    ids = torch.empty(T, topk, dtype=ids_dtype, device=dev)
    _lib.call("moe_topk_softmax", _ptr(logits), _code(logits), T, E, topk, int(renormalize),
              _ptr(w), _code(w), _ptr(ids), _code(ids), _stream(dev))
    return w, ids


def grouped_topk(hidden_states: torch.Tensor, gating_output: torch.Tensor, topk: int,
                 renormalize: bool, num_expert_group: int, topk_group: int,
                 scoring_func: str = "softmax", routed_scaling_factor: float = 1.0
                 ) -> tuple[torch.Tensor, torch.Tensor]:
    """Grouped top-k routing of kernels/track1-triton/groupedtopk/base.py:31-72
    in one kernel (moe_grouped_topk): softmax or sigmoid scores, the
    `topk_group` expert groups with the best maximum score, the top-k experts
    among them (descending, ties to the lower index), weights renormalised
    when asked and scaled by `routed_scaling_factor`. Returns (topk_weights
    fp32 [T, k], topk_ids int32 [T, k]) like the reference.
    """
    _check_cuda("gating_output", gating_output)
    if gating_output.dim() != 2 or gating_output.shape[0] != hidden_states.shape[0]:
        raise ValueError("gating_output must be [T, E] with T = hidden_states.shape[0]")
    if scoring_func not in ("softmax", "sigmoid"):
        raise ValueError(f"Unsupported scoring_func: {scoring_func}")
    logits = _contig(gating_output)
    T, E = logits.shape
    dev = logits.device
    w = torch.empty(T, topk, dtype=torch.float32, device=dev)
    ids = torch.empty(T, topk, dtype=torch.int32, device=dev)
    _lib.call("moe_grouped_topk", _ptr(logits), _code(logits), T, E, topk, int(renormalize),
              num_expert_group, topk_group, 0 if scoring_func == "softmax" else 1,
              float(routed_scaling_factor), _ptr(w), _ptr(ids), _stream(dev))
    return w, ids


# ---------------------------------------------------------------------------
# moe_align_block_size
# ---------------------------------------------------------------------------

def moe_align_block_size(topk_ids: torch.Tensor, block_size: int, num_experts: int
                         ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Groups flat (token, slot) indices by expert, padded to `block_size`.

    Returns (sorted_token_ids int32 [L], expert_ids int32 [L / block_size],
    num_tokens_post_pad int32 [1]) with L = moe_align_buffer_len. Within an
    expert the flat indices ascend (the row order of base.py's
    `x_rep[flat_ids == e]`); padding slots hold topk_ids.numel(); ids outside
    [0, num_experts) are dropped.
    """
    _check_cuda("topk_ids", topk_ids)
    ids = _contig(topk_ids)
    if ids.dtype not in (torch.int32, torch.int64):
        raise TypeError("topk_ids must be int32 or int64")
    lib = _lib.load()
    numel = ids.numel()
    L = lib.moe_align_buffer_len(numel, num_experts, block_size)
    if L < 0:
        raise ValueError("invalid align arguments")
    ws_bytes = ctypes.c_size_t(0)
    _lib.check(lib.moe_align_workspace_size(numel, num_experts, block_size,
                                            ctypes.byref(ws_bytes)), "moe_align_workspace_size")
    dev = ids.device
    sorted_ids = torch.empty(L, dtype=torch.int32, device=dev)
    expert_ids = torch.empty(L // block_size, dtype=torch.int32, device=dev)
    npp = torch.empty(1, dtype=torch.int32, device=dev)
    ws = _workspace(dev, ws_bytes.value) if ws_bytes.value else None
    _lib.call("moe_align_block_size", _ptr(ids), _code(ids), numel, num_experts, block_size,
              _ptr(sorted_ids), _ptr(expert_ids), _ptr(npp), _ptr(ws), ws_bytes.value,
              _stream(dev))
    return sorted_ids, expert_ids, npp


# ---------------------------------------------------------------------------
# Weight preparation (replaces the per-call casts of base.py:60-61)
# ---------------------------------------------------------------------------

@dataclass
class PreparedWeights:
    """Expert weights in the layout and format the grouped GEMMs read."""

    w13: torch.Tensor               # [E, 2I, H], gate/up rows regrouped by 16
    w2: torch.Tensor                # [E, H, I]
    w13_scale: torch.Tensor | None  # fp8: [E, 2I/128, H/128]; int8: [E, 2I]
    w2_scale: torch.Tensor | None   # fp8: [E, H/128, I/128];  int8: [E, H]
    #                                 fp8-ue8m0: uint8 scale-factor images
    quant: str                      # "none" | "fp8" | "int8" | "fp8-ue8m0"
    num_experts: int
    inter_size: int
    hidden_size: int

    @property
    def compute_dtype(self) -> torch.dtype:
        return self.w13.dtype


def compute_dtype_for(act_dtype: torch.dtype, quant: str = "none") -> torch.dtype:
    """Operand dtype of the expert GEMMs for activations of `act_dtype`: f16
    and bf16 compute in their own dtype; f32 activations keep f32 operands,
    multiplied as tf32 by the tensor cores, when the weights are unquantised
    (the W8A8 paths take bf16)."""
    if act_dtype == torch.float16:
        return torch.float16
    if act_dtype == torch.float32 and quant == "none":
        return torch.float32
    return torch.bfloat16


def prepare_weights(w1: torch.Tensor, w2: torch.Tensor, quant: str = "none",
                    compute_dtype: torch.dtype = torch.bfloat16,
                    w1_scale: torch.Tensor | None = None,
                    w2_scale: torch.Tensor | None = None) -> PreparedWeights:
    """Casts or quantises w1 [E, 2I, H] and w2 [E, H, I] once.

    quant "none": cast to `compute_dtype` (bf16, f16, or f32 for the tf32
    GEMMs of f32 activations; see compute_dtype_for). quant "fp8": e4m3
    with one fp32 scale per 128x128 block (absmax / 448), or pass-through of
    already-e4m3 weights with `w1_scale`/`w2_scale`. quant "int8": int8 with
    one scale per output row (absmax / 127). quant "fp8-ue8m0": e4m3 with one
    power-of-two scale per 128x128 block (the smallest with absmax / scale <=
    448), kept as the scale-factor images the tensor core reads
    (moe_ue8m0_scale_bytes layout); needs H and I divisible by 128.
    """
    _check_cuda("w1", w1)
    _check_cuda("w2", w2)
    if quant not in _QUANT:
        raise ValueError(f"quant must be one of {sorted(_QUANT)}")
    if w1.dim() != 3 or w2.dim() != 3:
        raise ValueError("w1 must be [E, 2I, H] and w2 [E, H, I]")
    E, two_i, H = w1.shape
    if two_i % 2 or w2.shape != (E, H, two_i // 2):
        raise ValueError(f"w2 shape {tuple(w2.shape)} does not match w1 {tuple(w1.shape)}")
    inter = two_i // 2
    w1c, w2c = _contig(w1.detach()), _contig(w2.detach())
    dev = w1.device
    q = _QUANT[quant]
    if quant == "none":
        if compute_dtype not in (torch.bfloat16, torch.float16, torch.float32):
            raise ValueError("compute_dtype must be bf16, f16 or f32")
        dst_dtype = compute_dtype
        s13 = s2 = None
    elif quant == "fp8":
        dst_dtype = torch.float8_e4m3fn
        s13 = torch.empty(E, -(-two_i // 128), -(-H // 128), dtype=torch.float32, device=dev)
        s2 = torch.empty(E, -(-H // 128), -(-inter // 128), dtype=torch.float32, device=dev)
    elif quant == "fp8-ue8m0":
        if H % 128 or inter % 128:
            raise ValueError("fp8-ue8m0 needs hidden and intermediate sizes divisible by 128")
        if w1c.dtype == torch.float8_e4m3fn:
            raise ValueError("fp8-ue8m0 quantises f32/f16/bf16 weights itself")
        dst_dtype = torch.float8_e4m3fn
        lib = _lib.load()
        s13 = torch.empty(lib.moe_ue8m0_scale_bytes(E, two_i, H), dtype=torch.uint8, device=dev)
        s2 = torch.empty(lib.moe_ue8m0_scale_bytes(E, H, inter), dtype=torch.uint8, device=dev)
    else:
        dst_dtype = torch.int8
        s13 = torch.empty(E, two_i, dtype=torch.float32, device=dev)
        s2 = torch.empty(E, H, dtype=torch.float32, device=dev)
    if w1c.dtype == torch.float8_e4m3fn and (w1_scale is None or w2_scale is None):
        raise ValueError("e4m3 weights need w1_scale and w2_scale")
    o13 = torch.empty(E, two_i, H, dtype=dst_dtype, device=dev)
    o2 = torch.empty(E, H, inter, dtype=dst_dtype, device=dev)
    st = _stream(dev)
    # the library takes every scale buffer as float* (UE8M0 images are bytes)
    sc1 = _contig(w1_scale.float()) if w1_scale is not None else None
    sc2 = _contig(w2_scale.float()) if w2_scale is not None else None
    _lib.call("moe_prepare_w13", _ptr(w1c), _code(w1c), _ptr(sc1), E, inter, H, q, _ptr(o13),
              _DTYPE_CODE[dst_dtype], _ptr(s13), st)
    _lib.call("moe_prepare_w2", _ptr(w2c), _code(w2c), _ptr(sc2), E, H, inter, q, _ptr(o2),
              _DTYPE_CODE[dst_dtype], _ptr(s2), st)
    return PreparedWeights(o13, o2, s13, s2, quant, E, inter, H)


_prep_lock = threading.Lock()
_prep_cache: dict = {}


def _cached_prepare(w1, w2, quant, compute_dtype, w1_scale, w2_scale) -> PreparedWeights:
    """prepare_weights memoised on the identity and version of the inputs.

    An entry holds weak references to the tensors it was made from and is
    used only while they still name those same tensor objects: once a
    source tensor is freed, a new tensor that the caching allocator places
    at the same address (same shape, version 0) does not match it."""
    srcs = (w1, w2, w1_scale, w2_scale)
    key = (w1.data_ptr(), w1._version, tuple(w1.shape), w1.dtype,
           w2.data_ptr(), w2._version, tuple(w2.shape), w2.dtype, quant, compute_dtype,
           None if w1_scale is None else (w1_scale.data_ptr(), w1_scale._version),
           None if w2_scale is None else (w2_scale.data_ptr(), w2_scale._version))
    with _prep_lock:
        hit = _prep_cache.get(key)
    if hit is not None:
        prep, refs = hit
        if all((r is None and t is None) or (r is not None and r() is t)
               for r, t in zip(refs, srcs)):
            return prep
    prep = prepare_weights(w1, w2, quant, compute_dtype, w1_scale, w2_scale)
    refs = tuple(None if t is None else weakref.ref(t) for t in srcs)
    with _prep_lock:
        if len(_prep_cache) > 8:
            _prep_cache.clear()
        _prep_cache[key] = (prep, refs)
    return prep


# ---------------------------------------------------------------------------
# fused_experts (base.py:50-76)
# ---------------------------------------------------------------------------

def _problem(hidden, prep: PreparedWeights, topk_weights, topk_ids, out, status,
             events_array=None, num_tokens_dev=None):
    p = _lib.MoeProblem()
    p.num_tokens = hidden.shape[0]
    p.hidden_size = prep.hidden_size
    p.inter_size = prep.inter_size
    p.num_experts = prep.num_experts
    p.top_k = topk_ids.shape[1]
    p.act_dtype = _code(hidden)
    p.quant = _QUANT[prep.quant]
    p.ids_dtype = _code(topk_ids)
    p.weights_dtype = _code(topk_weights)
    p.hidden = hidden.data_ptr()
    p.w13 = prep.w13.data_ptr()
    p.w2 = prep.w2.data_ptr()
    p.w13_scale = prep.w13_scale.data_ptr() if prep.w13_scale is not None else None
    p.w2_scale = prep.w2_scale.data_ptr() if prep.w2_scale is not None else None
    p.topk_weights = topk_weights.data_ptr()
    p.topk_ids = topk_ids.data_ptr()
    p.out = out.data_ptr()
    p.status = status.data_ptr() if status is not None else None
    p.stage_events = ctypes.cast(events_array, ctypes.c_void_p) if events_array is not None \
        else None
    p.num_tokens_dev = num_tokens_dev.data_ptr() if num_tokens_dev is not None else None
    return p


def fused_experts_launches(num_tokens: int, hidden_size: int, intermediate_size: int,
                           num_experts: int, top_k: int, quant: str = "none",
                           dtype: torch.dtype = torch.bfloat16, rows_only: bool = False) -> int:
    """Kernels one fused_experts call of this shape launches (the plan's
    answer, moe_fused_experts_launches; no GPU needed)."""
    p = _lib.MoeProblem()
    p.num_tokens = num_tokens
    p.hidden_size = hidden_size
    p.inter_size = intermediate_size
    p.num_experts = num_experts
    p.top_k = top_k
    p.act_dtype = _code(torch.empty(0, dtype=dtype))
    p.quant = _QUANT[quant]
    p.ids_dtype = _lib.DT_I32
    p.weights_dtype = _lib.DT_F32
    n = ctypes.c_int(0)
    _lib.call("moe_fused_experts_launches", ctypes.byref(p), int(rows_only), ctypes.byref(n))
    return n.value


def fused_moe_launches(num_tokens: int, hidden_size: int, intermediate_size: int,
                       num_experts: int, top_k: int, quant: str = "none",
                       dtype: torch.dtype = torch.bfloat16,
                       logits_dtype: torch.dtype = torch.float32) -> int:
    """Kernels fused_moe launches (moe_fused_moe_launches; answers without a
    GPU): fused_experts' launches plus the routing kernel, which the decode
    path does not need for fp32 logits over at most 256 experts (its first
    kernel routes the tokens itself)."""
    p = _lib.MoeProblem()
    p.num_tokens = num_tokens
    p.hidden_size = hidden_size
    p.inter_size = intermediate_size
    p.num_experts = num_experts
    p.top_k = top_k
    p.act_dtype = _code(torch.empty(0, dtype=dtype))
    p.quant = _QUANT[quant]
    p.ids_dtype = _lib.DT_I32
    p.weights_dtype = _code(torch.empty(0, dtype=dtype))
    n = ctypes.c_int(0)
    _lib.call("moe_fused_moe_launches", ctypes.byref(p),
              _code(torch.empty(0, dtype=logits_dtype)), ctypes.byref(n))
    return n.value


def fused_experts_plan(num_tokens: int, hidden_size: int, intermediate_size: int,
                       num_experts: int, top_k: int, quant: str = "none",
                       dtype: torch.dtype = torch.bfloat16) -> dict:
    """The tile widths and K splits fused_experts picks for this shape, and
    whether it gathers token by token or takes the decode kernels
    (moe_fused_experts_plan; no GPU needed)."""
    p = _lib.MoeProblem()
    p.num_tokens = num_tokens
    p.hidden_size = hidden_size
    p.inter_size = intermediate_size
    p.num_experts = num_experts
    p.top_k = top_k
    p.act_dtype = _code(torch.empty(0, dtype=dtype))
    p.quant = _QUANT[quant]
    p.ids_dtype = _lib.DT_I32
    p.weights_dtype = _lib.DT_F32
    info = (ctypes.c_int32 * 8)()
    _lib.call("moe_fused_experts_plan", ctypes.byref(p), info)
    keys = ("gate_up_block_n", "gate_up_splits", "down_block_n", "down_splits",
            "down_rows_dtype", "token_gather", "decode_path", "sms")
    return dict(zip(keys, list(info)))


def stage_event_array(events) -> ctypes.Array:
    """cudaEvent_t[7] for moe_problem_t.stage_events from torch.cuda.Event
    objects (each must have been recorded once so that it exists)."""
    if len(events) != len(_lib.STAGES) + 1:
        raise ValueError(f"need {len(_lib.STAGES) + 1} events")
    handles = [ev.cuda_event for ev in events]
    if any(h == 0 for h in handles):
        raise ValueError("record each event once before passing it")
    return (ctypes.c_void_p * len(handles))(*handles)


def fused_experts(hidden_states: torch.Tensor, w1, w2: torch.Tensor | None,
                  topk_weights: torch.Tensor, topk_ids: torch.Tensor,
                  activation: str = "silu", use_fp8_w8a8: bool = False,
                  use_int8_w8a8: bool = False, w1_scale: torch.Tensor | None = None,
                  w2_scale: torch.Tensor | None = None, a1_scale: torch.Tensor | None = None,
                  a2_scale: torch.Tensor | None = None, block_shape: list[int] | None = None,
                  out: torch.Tensor | None = None, status: torch.Tensor | None = None,
                  stage_events: ctypes.Array | None = None,
                  rows_only: bool = False, scale_format: str | None = None,
                  router_logits: torch.Tensor | None = None,
                  renormalize: bool = True,
                  num_tokens_dev: torch.Tensor | None = None) -> torch.Tensor:
    """out[t] = sum_j w[t,j] * W2[e] (silu(W1g[e] x_t) * W1u[e] x_t), e = ids[t,j].

    scale_format (fp8 only): "ue8m0" (block scales rounded up to a power of
    two, absmax / 448 <= scale < 2 * absmax / 448, applied by the tensor
    core; weights prepared with quant "fp8-ue8m0") or "fp32" (scale = absmax
    / 448 exactly, applied per k-block in the epilogue). The default (None)
    is "ue8m0" for f32/f16/bf16 weights whose hidden and intermediate sizes
    are multiples of 128 -- the faster kernel, at the same accuracy against
    the unquantised layer -- and "fp32" for weights given already quantised
    to e4m3 with their fp32 block scales.

    router_logits [T, E] (f32/f16/bf16): route inside the same library call
    (moe_fused_moe): topk_weights and topk_ids are then OUTPUT buffers [T, k]
    that the routing of base.py:44-48 fills (softmax in fp32, top-k,
    renormalised when `renormalize`).

    num_tokens_dev: a one-element int32 CUDA tensor; only the first
    num_tokens_dev[0] tokens take part and the other rows of `out` are left
    untouched (an expert-parallel receive buffer, sized for the worst case,
    processed at the size it got without a host sync).

    rows_only (top_k == 1): rows of tokens whose expert id is dropped are left
    unspecified instead of zeroed, which lets the down GEMM write the result
    rows directly (moe_fused_experts_rows; the expert-parallel receive buffer).

    hidden_states [T, H] (f32/f16/bf16); w1 [E, 2I, H] and w2 [E, H, I] raw
    (cast or quantised once and cached) or `w1` a PreparedWeights and `w2`
    None; topk_weights [T, k] (f32/f16/bf16); topk_ids [T, k] (int32/int64).
    Activations are quantised dynamically in the W8A8 modes (fp8: per token
    per 128 columns; int8: per token). Returns [T, H] in hidden_states.dtype.
    """
    if activation != "silu":
        raise ValueError(f"unsupported activation {activation!r}; the operator is SiLU-gated")
    if a1_scale is not None or a2_scale is not None:
        raise NotImplementedError("static activation scales are not supported; "
                                  "activations are quantised per token")
    if use_fp8_w8a8 and use_int8_w8a8:
        raise ValueError("choose one of use_fp8_w8a8 / use_int8_w8a8")
    if use_fp8_w8a8 and block_shape is not None and list(block_shape) != [128, 128]:
        raise ValueError("fp8 W8A8 supports block_shape [128, 128] only")
    _check_cuda("hidden_states", hidden_states)
    _check_cuda("topk_weights", topk_weights)
    _check_cuda("topk_ids", topk_ids)
    if hidden_states.dim() != 2 or topk_ids.dim() != 2 or topk_weights.shape != topk_ids.shape:
        raise ValueError("expected hidden_states [T, H], topk_weights/topk_ids [T, k]")
    if topk_ids.shape[0] != hidden_states.shape[0]:
        raise ValueError("topk_ids and hidden_states disagree on the token count")
    if scale_format not in (None, "fp32", "ue8m0"):
        raise ValueError("scale_format must be None, 'fp32' or 'ue8m0'")
    quant = "fp8" if use_fp8_w8a8 else ("int8" if use_int8_w8a8 else "none")
    if quant == "fp8" and scale_format is None and not isinstance(w1, PreparedWeights):
        raw = w1.dtype in (torch.float32, torch.float16, torch.bfloat16)
        sizes = w1.dim() == 3 and w1.shape[1] % 256 == 0 and w1.shape[2] % 128 == 0
        scale_format = "ue8m0" if raw and sizes and w1_scale is None else "fp32"
    if quant == "fp8" and scale_format == "ue8m0":
        quant = "fp8-ue8m0"
    compute = compute_dtype_for(hidden_states.dtype, quant)
    if isinstance(w1, PreparedWeights):
        prep = w1
        if quant == "fp8" and prep.quant == "fp8-ue8m0":
            quant = prep.quant  # prepared fp8 weights carry their scale format
        if prep.quant != quant:
            raise ValueError(f"prepared weights are {prep.quant!r}, call asked for {quant!r}")
        if quant == "none" and prep.compute_dtype != compute:
            raise ValueError("prepared weights dtype does not match the activation dtype")
    else:
        _check_cuda("w1", w1)
        _check_cuda("w2", w2)
        prep = _cached_prepare(w1, w2, quant, compute, w1_scale, w2_scale)
    T, H = hidden_states.shape
    if H != prep.hidden_size:
        raise ValueError(f"hidden size {H} does not match the weights ({prep.hidden_size})")
    hidden = _contig(hidden_states)
    tw = _contig(topk_weights)
    ti = _contig(topk_ids)
    if out is None:
        out = torch.empty_like(hidden)
    elif (out.shape != hidden.shape or out.dtype != hidden.dtype or not out.is_contiguous()
          or out.data_ptr() % 16):
        raise ValueError("out must be a contiguous, 16-byte aligned tensor like hidden_states")
    if num_tokens_dev is not None:
        _check_cuda("num_tokens_dev", num_tokens_dev)
        if num_tokens_dev.dtype != torch.int32 or num_tokens_dev.numel() < 1:
            raise ValueError("num_tokens_dev must be an int32 CUDA tensor with one element")
    p = _problem(hidden, prep, tw, ti, out, status, stage_events, num_tokens_dev)
    lib = _lib.load()
    nbytes = ctypes.c_size_t(0)
    _lib.check(lib.moe_fused_experts_workspace_size(ctypes.byref(p), ctypes.byref(nbytes)),
               "moe_fused_experts_workspace_size")
    ws = _workspace(hidden.device, nbytes.value)
    if router_logits is not None:
        if rows_only:
            raise ValueError("rows_only takes routed ids, not router logits")
        _check_cuda("router_logits", router_logits)
        logits = _contig(router_logits)
        if logits.shape != (T, prep.num_experts):
            raise ValueError(f"router_logits must be [T, E] = [{T}, {prep.num_experts}]")
        if tw.data_ptr() != topk_weights.data_ptr() or ti.data_ptr() != topk_ids.data_ptr():
            raise ValueError("topk_weights / topk_ids receive the routing: pass dense, "
                             "16-byte aligned tensors")
        _lib.check(lib.moe_fused_moe(ctypes.byref(p), _ptr(logits), _code(logits),
                                     int(bool(renormalize)), _ptr(ws), ws.numel(),
                                     _stream(hidden.device)), "moe_fused_moe")
        return out
    entry = "moe_fused_experts_rows" if rows_only else "moe_fused_experts"
    _lib.check(getattr(lib, entry)(ctypes.byref(p), _ptr(ws), ws.numel(),
                                   _stream(hidden.device)), entry)
    return out


def fused_moe(hidden_states: torch.Tensor, w1, w2, gating_output: torch.Tensor, topk: int,
              renormalize: bool = True, **kwargs) -> torch.Tensor:
    """Routing + experts: the whole of base.py:35-76 as one library call
    (moe_fused_moe). The routing weights are rounded to the activation dtype
    before use, as base.py:48 casts them; the result equals fused_topk
    followed by fused_experts bit for bit."""
    _check_cuda("hidden_states", hidden_states)
    T = hidden_states.shape[0]
    dev = hidden_states.device
    topk_weights = torch.empty(T, topk, dtype=hidden_states.dtype, device=dev)
    topk_ids = torch.empty(T, topk, dtype=torch.int32, device=dev)
    return fused_experts(hidden_states, w1, w2, topk_weights, topk_ids,
                         router_logits=gating_output, renormalize=renormalize, **kwargs)


# ---------------------------------------------------------------------------
# Drop-in module (base.py:8-76)
# ---------------------------------------------------------------------------

class ModelNew(nn.Module):
    """Same constructor, parameters and forward contract as base.py's Model."""

    def __init__(self, num_experts: int, top_k: int, hidden_size: int,
                 intermediate_size: int, renormalize: bool = True):
        super().__init__()
        self.num_experts = num_experts
        self.top_k = top_k
        self.hidden_size = hidden_size
        self.intermediate_size = intermediate_size
        self.renormalize = renormalize
        self.w1 = nn.Parameter(torch.empty(num_experts, 2 * intermediate_size, hidden_size))
        self.w2 = nn.Parameter(torch.empty(num_experts, hidden_size, intermediate_size))
        nn.init.normal_(self.w1, std=0.02)
        nn.init.normal_(self.w2, std=0.02)
        # not a buffer: load_state_dict(strict=True) must see only w1/w2
        self._prepared: dict = {}

    def prepared(self, act_dtype: torch.dtype, quant: str = "none") -> PreparedWeights:
        """The prepared weights for this activation dtype, made once per
        weight version. An entry also holds weak references to the w1/w2
        objects it was made from, so a parameter replaced by a new tensor
        that happens to reuse the old address (version 0 again) is
        prepared afresh instead of matching the stale entry."""
        compute = compute_dtype_for(act_dtype, quant)
        w1, w2 = self.w1, self.w2
        key = (quant, compute, w1.data_ptr(), w1._version, tuple(w1.shape), w1.dtype,
               w2.data_ptr(), w2._version, tuple(w2.shape), w2.dtype)
        hit = self._prepared.get(key)
        if hit is not None:
            prep, r1, r2 = hit
            if r1() is w1 and r2() is w2:
                return prep
        self._prepared.clear()
        prep = prepare_weights(w1, w2, quant, compute)
        self._prepared[key] = (prep, weakref.ref(w1), weakref.ref(w2))
        return prep

    def forward(self, hidden_states: torch.Tensor, router_logits: torch.Tensor) -> torch.Tensor:
        self._last_hidden = hidden_states  # for run_out (auto_bench kernel profiling)
        # routing + experts in one library call; the routing weights are in
        # the activation dtype, as base.py:48 casts them
        return fused_moe(hidden_states, self.prepared(hidden_states.dtype), None, router_logits,
                         self.top_k, self.renormalize)

    def run_out(self, router_logits: torch.Tensor, out: torch.Tensor,
                hidden_states: torch.Tensor | None = None) -> torch.Tensor:
        """auto_bench `--profile-mode kernel` hook: forward into `out`."""
        hidden = hidden_states if hidden_states is not None else self._last_hidden
        return fused_moe(hidden, self.prepared(hidden.dtype), None, router_logits, self.top_k,
                         self.renormalize, out=out)


# ---------------------------------------------------------------------------
# CUDA-graph capture for a fixed token count (decode loops)
# ---------------------------------------------------------------------------

class CapturedMoE:
    """Routing + fused experts for a fixed token count, captured once in a CUDA
    graph and replayed: one graph launch instead of 6-8 kernel launches, which
    is what bounds decode-sized batches.

    `fn(hidden, logits) -> out` is the forward to capture (e.g. a ModelNew);
    it must not synchronise the host. Inputs are copied into static buffers
    (`hidden`, `logits` attributes; write them directly to skip the copies);
    the returned tensor is the static output buffer, overwritten by the next
    replay.
    """

    def __init__(self, fn, num_tokens: int, hidden_size: int, num_experts: int,
                 dtype: torch.dtype = torch.bfloat16, device=None, warmup: int = 2):
        dev = torch.device(device) if device is not None else torch.device(
            "cuda", torch.cuda.current_device())
        self.fn = fn
        self.hidden = torch.zeros(num_tokens, hidden_size, dtype=dtype, device=dev)
        self.logits = torch.zeros(num_tokens, num_experts, dtype=torch.float32, device=dev)
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side), torch.no_grad():
            for _ in range(warmup):  # one-time setup (weights, attributes) off the capture
                fn(self.hidden, self.logits)
        torch.cuda.current_stream(dev).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph), torch.no_grad():
            self.out = fn(self.hidden, self.logits)

    def replay(self) -> torch.Tensor:
        self.graph.replay()
        return self.out

    def __call__(self, hidden_states: torch.Tensor, router_logits: torch.Tensor) -> torch.Tensor:
        self.hidden.copy_(hidden_states, non_blocking=True)
        self.logits.copy_(router_logits, non_blocking=True)
        return self.replay()


class GroupedTopK(nn.Module):
    """Drop-in for kernels/track1-triton/groupedtopk/base.py's Model: same
    constructor and forward(hidden_states, gating_output) -> (topk_weights
    fp32 [T, k], topk_ids int32 [T, k]), computed by one kernel."""

    def __init__(self, topk: int, renormalize: bool, num_expert_group: int, topk_group: int,
                 scoring_func: str = "softmax", routed_scaling_factor: float = 1.0):
        super().__init__()
        if scoring_func not in ("softmax", "sigmoid"):
            raise ValueError(f"Unsupported scoring_func: {scoring_func}")
        self.topk = topk
        self.renormalize = renormalize
        self.num_expert_group = num_expert_group
        self.topk_group = topk_group
        self.scoring_func = scoring_func
        self.routed_scaling_factor = routed_scaling_factor

    def forward(self, hidden_states: torch.Tensor, gating_output: torch.Tensor):
        if hidden_states.size(0) != gating_output.size(0):
            raise ValueError("hidden_states and gating_output disagree on the token count")
        return grouped_topk(hidden_states, gating_output, self.topk, self.renormalize,
                            self.num_expert_group, self.topk_group, self.scoring_func,
                            self.routed_scaling_factor)


class HostPipeline:
    """Forwards over host (pinned) inputs with the copies of consecutive calls
    overlapped: while the compute stream runs step i, a copy stream brings in
    step i+1's inputs and another takes out step i-1's output. Device staging
    buffers are double-buffered and handed between the streams with events.

    `fn(hidden, logits) -> out` is the forward (a ModelNew, a CapturedMoE, an
    expert-parallel step ...). `submit(hidden_host, logits_host, out_host)`
    enqueues one step and returns at once; `out_host` holds that step's
    output after `flush()` (or any later synchronisation). Work is ordered
    after whatever the caller's current stream had enqueued when `submit` was
    called, and `flush()` makes the caller's current stream wait for all of it.
    """

    def __init__(self, fn, num_tokens: int, hidden_size: int, num_experts: int,
                 dtype: torch.dtype = torch.bfloat16, device=None, out_dtype=None):
        dev = torch.device(device) if device is not None else torch.device(
            "cuda", torch.cuda.current_device())
        self.fn = fn
        self.device = dev
        self.h = [torch.empty(num_tokens, hidden_size, dtype=dtype, device=dev) for _ in range(2)]
        self.l = [torch.empty(num_tokens, num_experts, dtype=torch.float32, device=dev)
                  for _ in range(2)]
        self.o = [torch.empty(num_tokens, hidden_size, dtype=out_dtype or dtype, device=dev)
                  for _ in range(2)]
        self.copy_in = torch.cuda.Stream(dev)
        self.compute = torch.cuda.Stream(dev)
        self.copy_out = torch.cuda.Stream(dev)
        self.ev_in = [torch.cuda.Event() for _ in range(2)]      # inputs of slot landed
        self.ev_used = [torch.cuda.Event() for _ in range(2)]    # compute done with inputs
        self.ev_done = [torch.cuda.Event() for _ in range(2)]    # output staged
        self.ev_taken = [torch.cuda.Event() for _ in range(2)]   # output copied out
        for evs in (self.ev_used, self.ev_taken):
            for ev in evs:
                ev.record(torch.cuda.current_stream(dev))
        self.i = 0

    def submit(self, hidden_host: torch.Tensor, logits_host: torch.Tensor,
               out_host: torch.Tensor) -> None:
        slot = self.i % 2
        self.i += 1
        caller = torch.cuda.current_stream(self.device)
        self.copy_in.wait_stream(caller)
        self.copy_in.wait_event(self.ev_used[slot])
        with torch.cuda.stream(self.copy_in):
            self.h[slot].copy_(hidden_host, non_blocking=True)
            self.l[slot].copy_(logits_host, non_blocking=True)
            self.ev_in[slot].record(self.copy_in)
        self.compute.wait_event(self.ev_in[slot])
        self.compute.wait_event(self.ev_taken[slot])
        with torch.cuda.stream(self.compute), torch.no_grad():
            out = self.fn(self.h[slot], self.l[slot])
            self.ev_used[slot].record(self.compute)
            self.o[slot].copy_(out)
            self.ev_done[slot].record(self.compute)
        self.copy_out.wait_event(self.ev_done[slot])
        with torch.cuda.stream(self.copy_out):
            out_host.copy_(self.o[slot], non_blocking=True)
            self.ev_taken[slot].record(self.copy_out)

    def flush(self) -> None:
        """Makes the caller's current stream wait for every submitted step."""
        caller = torch.cuda.current_stream(self.device)
        caller.wait_stream(self.copy_out)
        caller.wait_stream(self.compute)
