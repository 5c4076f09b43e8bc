"""ctypes binding of libmoe_b200.so, the C ABI declared in include/moe_b200.h.

The library is loaded from kernelswift_b200/lib/ (built in-tree by
`python -m kernelswift_b200.build`). There is no fallback: if the library is
missing or fails to load, every operator raises.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libmoe_b200.so"

# moe_status_t
MOE_OK = 0
MOE_ERR_INVALID_ARG = 1
MOE_ERR_UNSUPPORTED = 2
MOE_ERR_CUDA = 3
MOE_ERR_TIMEOUT = 4
MOE_ERR_WORKSPACE = 5
MOE_ERR_DEVICE = 6

# moe_dtype_t
DT_F32, DT_F16, DT_BF16, DT_E4M3, DT_I8, DT_I32, DT_I64 = range(7)

# moe_quant_t
QUANT_NONE, QUANT_FP8_BLOCK, QUANT_INT8_CHANNEL, QUANT_FP8_UE8M0 = range(4)

_vp = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64
_int = ctypes.c_int
_sz = ctypes.c_size_t
_fp = ctypes.POINTER(ctypes.c_float)


class MoeProblem(ctypes.Structure):
    """Mirror of moe_problem_t."""

    _fields_ = [
        ("num_tokens", _i64),
        ("hidden_size", _i64),
        ("inter_size", _i64),
        ("num_experts", _i32),
        ("top_k", _i32),
        ("act_dtype", _i32),
        ("quant", _i32),
        ("ids_dtype", _i32),
        ("weights_dtype", _i32),
        ("hidden", _vp),
        ("w13", _vp),
        ("w2", _vp),
        ("w13_scale", _vp),
        ("w2_scale", _vp),
        ("topk_weights", _vp),
        ("topk_ids", _vp),
        ("out", _vp),
        ("status", _vp),
        ("stage_events", _vp),
        ("num_tokens_dev", _vp),
    ]


# Stages of moe_fused_experts (stage_events indices)
STAGES = ("align", "gather", "gate_up", "quant", "down", "sum")


# name -> (restype, argtypes); one entry per declaration of include/moe_b200.h
SIGNATURES = {
    "moe_status_string": (ctypes.c_char_p, [_int]),
    "moe_last_error": (ctypes.c_char_p, []),
    "moe_abi_version": (_int, []),
    "moe_read_status": (_int, [_vp, _vp, _int, _vp]),
    "moe_topk_softmax": (_int, [_vp, _int, _i64, _int, _int, _int, _vp, _int, _vp, _int, _vp]),
    "moe_align_buffer_len": (_i64, [_i64, _int, _int]),
    "moe_ue8m0_scale_bytes": (_i64, [_i64, _i64, _i64]),
    "moe_align_workspace_size": (_int, [_i64, _int, _int, ctypes.POINTER(_sz)]),
    "moe_align_block_size": (_int, [_vp, _int, _i64, _int, _int, _vp, _vp, _vp, _vp, _sz, _vp]),
    "moe_align_block_size_noalloc": (_int, [_vp, _int, _i64, _int, _int, _vp, _vp, _vp, _vp]),
    "moe_prepare_w13": (_int, [_vp, _int, _vp, _i64, _i64, _i64, _int, _vp, _int, _vp, _vp]),
    "moe_prepare_w2": (_int, [_vp, _int, _vp, _i64, _i64, _i64, _int, _vp, _int, _vp, _vp]),
    "moe_fused_experts_workspace_size": (_int, [ctypes.POINTER(MoeProblem), ctypes.POINTER(_sz)]),
    "moe_fused_experts": (_int, [ctypes.POINTER(MoeProblem), _vp, _sz, _vp]),
    "moe_fused_experts_rows": (_int, [ctypes.POINTER(MoeProblem), _vp, _sz, _vp]),
    "moe_fused_moe": (_int, [ctypes.POINTER(MoeProblem), _vp, _int, _int, _vp, _sz, _vp]),
    "moe_fused_experts_launches": (_int, [ctypes.POINTER(MoeProblem), _int,
                                          ctypes.POINTER(_int)]),
    "moe_fused_moe_launches": (_int, [ctypes.POINTER(MoeProblem), _int, ctypes.POINTER(_int)]),
    "moe_fused_experts_plan": (_int, [ctypes.POINTER(MoeProblem), _vp]),
    "moe_gather_rows": (_int, [_vp, _int, _i64, _i64, _int, _vp, _vp, _i64, _i64, _int, _vp,
                               _int, _vp, _vp]),
    "moe_gemm_gate_up": (_int, [_int, _int, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _int,
                                _i64, _i64, _vp, _int, _vp, _vp]),
    "moe_gemm_down": (_int, [_int, _int, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _int,
                             _i64, _i64, _vp, _int, _int, _vp, _int, _vp, _vp]),
    "moe_sum_topk": (_int, [_vp, _int, _i64, _int, _i64, _vp, _int, _int, _vp, _int, _vp]),
    "moe_ep_plan": (_int, [_vp, _int, _i64, _int, _int, _vp, _vp, _vp, _vp, _vp]),
    "moe_ep_plan_workspace_size": (_int, [_i64, _int, ctypes.POINTER(_sz)]),
    "moe_ep_plan_ws": (_int, [_vp, _int, _i64, _int, _int, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "moe_ep_plan_dedup": (_int, [_vp, _int, _vp, _int, _i64, _int, _int, _int, _vp, _vp, _vp,
                                 _vp, _vp, _vp]),
    "moe_grouped_topk": (_int, [_vp, _int, _i64, _int, _int, _int, _int, _int, _int,
                                ctypes.c_float, _vp, _vp, _vp]),
    "moe_combine_rows": (_int, [_vp, _int, _vp, _vp, _int, _i64, _int, _i64, _vp, _int, _vp]),
    "moe_selftest_wait_timeout": (_int, [_vp, _int, _vp]),
    "moe_selftest_sf_copy": (_int, [_vp, _vp, _vp, _vp]),
    "moe_ep_peer_create": (_int, [_int, _int, _i64, _i64, _int, _int, _int, _vp, _vp]),
    "moe_ep_peer_connect": (_int, [_vp, _vp]),
    "moe_ep_peer_buffers": (_int, [_vp, _vp, _vp, _vp, _vp, _vp]),
    "moe_ep_peer_dispatch": (_int, [_vp, _vp, _i64, _vp, _vp, _vp, _vp, _vp, _vp]),
    "moe_ep_peer_combine": (_int, [_vp, _vp, _i64, _vp, _vp, _vp]),
    "moe_ep_peer_disconnect": (_int, [_vp]),
    "moe_ep_peer_destroy": (_int, [_vp]),
}

EP_MAX_RANKS = 8
EP_HANDLE_BYTES = 64


class MoeError(RuntimeError):
    """A non-OK moe_status_t returned by the library."""

    def __init__(self, status: int, func: str, detail: str):
        self.status = status
        super().__init__(f"{func} failed: {status_name(status)}: {detail}")


_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Loads the library once and declares every entry point."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"{LIB_PATH} is missing; build it with `python -m kernelswift_b200.build`")
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def status_name(status: int) -> str:
    return load().moe_status_string(status).decode()


def check(status: int, func: str) -> None:
    if status != MOE_OK:
        detail = load().moe_last_error().decode()
        raise MoeError(status, func, detail)


def call(name: str, *args) -> None:
    """Calls an entry point that returns moe_status_t and raises on failure."""
    check(getattr(load(), name)(*args), name)
