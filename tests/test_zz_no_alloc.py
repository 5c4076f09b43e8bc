"""GPU: moe_align_block_size_noalloc, the variant for callers that cannot
allocate device memory (a runtime that owns all free HBM and offers no
workspace, or a path that must not risk cudaMalloc's device sync).

Its scratch is a static 1 MiB device array shared by every call. Each case
runs it twice in a row with different inputs, through the C ABI, and checks
both results bit for bit against moe_align_block_size with a caller-owned
workspace (integer routing metadata: exact equality is the tolerance).
"""
import ctypes

import pytest
import torch

from kernelswift_b200 import _lib

pytestmark = pytest.mark.gpu

SCRATCH_BYTES = 1 << 20


def ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def outputs(numel, E, bm, dev):
    L = _lib.load().moe_align_buffer_len(numel, E, bm)
    return (torch.full((L,), -7, dtype=torch.int32, device=dev),
            torch.full((L // bm,), -7, dtype=torch.int32, device=dev),
            torch.full((1,), -7, dtype=torch.int32, device=dev))


def with_workspace(ids, E, bm):
    lib = _lib.load()
    n = ctypes.c_size_t(0)
    _lib.check(lib.moe_align_workspace_size(ids.numel(), E, bm, ctypes.byref(n)),
               "moe_align_workspace_size")
    ws = torch.empty(max(n.value, 1), dtype=torch.uint8, device=ids.device)
    s, e, c = outputs(ids.numel(), E, bm, ids.device)
    code = _lib.DT_I64 if ids.dtype == torch.int64 else _lib.DT_I32
    _lib.call("moe_align_block_size", ptr(ids), code, ids.numel(), E, bm, ptr(s), ptr(e), ptr(c),
              ptr(ws), n.value, stream())
    return s, e, c


def no_alloc(ids, E, bm):
    s, e, c = outputs(ids.numel(), E, bm, ids.device)
    code = _lib.DT_I64 if ids.dtype == torch.int64 else _lib.DT_I32
    _lib.call("moe_align_block_size_noalloc", ptr(ids), code, ids.numel(), E, bm, ptr(s), ptr(e),
              ptr(c), stream())
    return s, e, c


def routed_ids(T, k, E, seed, dev, dtype=torch.int64):
    g = torch.Generator().manual_seed(seed)
    logits = torch.randn(T, E, generator=g) + torch.randn(E, generator=g)
    return torch.topk(logits, k, dim=-1).indices.to(dtype).to(dev)


CASES = [
    # (T, k, E, block_m): single-CTA path (no scratch), multi-CTA paths, and a
    # problem that fills most of the static scratch (1000 chunks x 256 experts).
    # The no-alloc entry partitions the ids into chunks of 4096 (single CTA up
    # to 8192), the workspace entry into chunks of 1024: equal outputs also
    # show the result does not depend on the partition.
    (37, 8, 32, 128),
    (8192, 8, 128, 128),
    (16384, 2, 8, 64),
    (512000, 8, 256, 128),
]


@pytest.mark.parametrize("T,k,E,bm", CASES)
def test_noalloc_matches_workspace_entry_point_twice(cuda_device, T, k, E, bm):
    for call, seed in enumerate((T, T + 1)):  # two calls in a row, different inputs
        ids = routed_ids(T, k, E, seed, cuda_device,
                         torch.int64 if call == 0 else torch.int32)
        want = with_workspace(ids, E, bm)
        got = no_alloc(ids, E, bm)
        torch.cuda.synchronize()
        for w, g in zip(want, got):
            assert torch.equal(w, g), (T, k, E, bm, call)


def test_noalloc_rejects_problems_beyond_the_static_scratch(cuda_device):
    E, numel = 1024, 2_000_000  # 489 chunks x 1024 experts x 4 B > 1 MiB
    ids = torch.zeros(numel, dtype=torch.int32, device=cuda_device)
    s, e, c = outputs(numel, E, 128, cuda_device)
    lib = _lib.load()
    st = lib.moe_align_block_size_noalloc(ptr(ids), _lib.DT_I32, numel, E, 128, ptr(s), ptr(e),
                                          ptr(c), stream())
    assert st == _lib.MOE_ERR_UNSUPPORTED
    assert "static scratch" in lib.moe_last_error().decode()
    torch.cuda.synchronize()
    assert int(c.item()) == -7  # nothing was launched
