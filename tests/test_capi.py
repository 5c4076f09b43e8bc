"""CPU tests of the C ABI: the library loads, exports every function that
include/*.h declares, and answers size queries without a GPU."""
import ctypes
import os
import re
from pathlib import Path

import pytest

from kernelswift_b200 import _lib
from oracle import moe_oracle as orc

ROOT = Path(__file__).resolve().parent.parent


def header_functions():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        for m in re.finditer(r"^\s*[A-Za-z_][\w\s\*]*?\b(moe_\w+)\s*\(", text, flags=re.M):
            names.add(m.group(1))
    return names


def test_header_parsed():
    names = header_functions()
    assert {"moe_align_block_size", "moe_fused_experts", "moe_gemm_gate_up"} <= names


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    missing = [n for n in sorted(header_functions()) if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_header():
    assert header_functions() == set(_lib.SIGNATURES)


def test_status_strings_and_version():
    lib = _lib.load()
    assert lib.moe_abi_version() == 2
    assert _lib.status_name(_lib.MOE_OK) == "MOE_OK"
    assert _lib.status_name(_lib.MOE_ERR_TIMEOUT) == "MOE_ERR_TIMEOUT"
    assert _lib.status_name(12345) == "MOE_ERR_UNKNOWN"


@pytest.mark.parametrize("numel,E,bm", [(0, 8, 16), (1, 8, 128), (166, 8, 128),
                                        (65536, 256, 128), (512, 256, 64)])
def test_align_buffer_len_matches_oracle(numel, E, bm):
    assert _lib.load().moe_align_buffer_len(numel, E, bm) == orc.align_buffer_len(numel, E, bm)


def test_align_workspace_query_rejects_bad_args():
    lib = _lib.load()
    n = ctypes.c_size_t(0)
    assert lib.moe_align_workspace_size(100, 8, 128, ctypes.byref(n)) == _lib.MOE_OK
    assert lib.moe_align_workspace_size(100, 0, 128, ctypes.byref(n)) == _lib.MOE_ERR_UNSUPPORTED
    assert lib.moe_align_workspace_size(100, 8, 100, ctypes.byref(n)) == _lib.MOE_ERR_UNSUPPORTED
    assert lib.moe_align_workspace_size(10 ** 6, 256, 128, ctypes.byref(n)) == _lib.MOE_OK
    assert n.value > 0  # the multi-CTA path needs per-chunk histograms


def test_fused_workspace_query_without_gpu():
    lib = _lib.load()
    p = _lib.MoeProblem()
    p.num_tokens, p.hidden_size, p.inter_size = 4096, 4096, 14336
    p.num_experts, p.top_k = 8, 2
    p.act_dtype, p.quant = _lib.DT_BF16, _lib.QUANT_NONE
    p.ids_dtype, p.weights_dtype = _lib.DT_I64, _lib.DT_BF16
    n = ctypes.c_size_t(0)
    assert lib.moe_fused_experts_workspace_size(ctypes.byref(p), ctypes.byref(n)) == _lib.MOE_OK
    L = orc.align_buffer_len(4096 * 2, 8, 128)
    assert n.value >= L * 4096 * 2 + L * 14336 * 2
    p.hidden_size = 100  # not a multiple of 64
    assert lib.moe_fused_experts_workspace_size(ctypes.byref(p), ctypes.byref(n)) \
        == _lib.MOE_ERR_UNSUPPORTED
    assert "hidden_size" in lib.moe_last_error().decode()


def test_compute_entry_points_fail_cleanly_without_gpu():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    lib = _lib.load()
    st = lib.moe_align_block_size(None, _lib.DT_I32, 0, 8, 128, None, None, None, None, 0, None)
    assert st in (_lib.MOE_ERR_CUDA, _lib.MOE_ERR_DEVICE)
    with pytest.raises(_lib.MoeError):
        _lib.call("moe_selftest_wait_timeout", None, 10, None)


def test_fused_experts_refuses_misaligned_operands():
    """A pointer off a 16-byte boundary is refused on the host, before any
    device call (the pointers here are never dereferenced)."""
    lib = _lib.load()

    def problem(quant=_lib.QUANT_NONE, **ptr):
        p = _lib.MoeProblem()
        p.num_tokens, p.hidden_size, p.inter_size = 64, 512, 256
        p.num_experts, p.top_k = 8, 2
        p.act_dtype, p.quant = _lib.DT_BF16, quant
        p.ids_dtype, p.weights_dtype = _lib.DT_I32, _lib.DT_BF16
        for name in ("hidden", "w13", "w2", "topk_weights", "topk_ids", "out"):
            setattr(p, name, ptr.get(name, 0x10000))
        if quant != _lib.QUANT_NONE:
            p.w13_scale = ptr.get("w13_scale", 0x20000)
            p.w2_scale = ptr.get("w2_scale", 0x20000)
        return p

    ws = ctypes.c_void_p(0x30000)
    for field in ("hidden", "w13", "w2", "out"):
        p = problem(**{field: 0x10008})
        assert lib.moe_fused_experts(ctypes.byref(p), ws, 1 << 30, None) \
            == _lib.MOE_ERR_INVALID_ARG, field
        assert "16-byte aligned" in lib.moe_last_error().decode()
    p = problem()
    assert lib.moe_fused_experts(ctypes.byref(p), ctypes.c_void_p(0x30004), 1 << 30, None) \
        == _lib.MOE_ERR_INVALID_ARG
    # int8 per-channel scales are read as float4; fp8 block scales one float at a time
    p = problem(_lib.QUANT_INT8_CHANNEL, w2_scale=0x20004)
    assert lib.moe_fused_experts(ctypes.byref(p), ws, 1 << 30, None) == _lib.MOE_ERR_INVALID_ARG
    p = problem(_lib.QUANT_FP8_BLOCK, w2_scale=0x20004)
    assert lib.moe_fused_experts(ctypes.byref(p), ws, 1 << 30, None) != _lib.MOE_ERR_INVALID_ARG


def test_python_wrapper_copies_misaligned_views():
    """fused_moe hands the library only 16-byte aligned dense tensors: an
    aligned dense tensor passes through, a view starting mid-vector or a
    strided view is copied."""
    import torch

    from kernelswift_b200 import fused_moe as fm

    base = torch.zeros(4 * 64 + 8, dtype=torch.bfloat16)
    assert base.data_ptr() % 16 == 0
    assert fm._contig(base) is base
    off = base[1:1 + 4 * 64].view(4, 64)  # starts 2 bytes past a boundary
    got = fm._contig(off)
    assert got is not off and got.data_ptr() % 16 == 0 and torch.equal(got, off)
    strided = base[:256].view(64, 4).t()
    got = fm._contig(strided)
    assert got.is_contiguous() and torch.equal(got, strided)


def test_prepared_weights_cache_checks_the_source_tensors(monkeypatch):
    """fused_experts' prepared-weight cache answers only for the very tensors
    (and versions) it prepared: another tensor object at the same address
    (here a view; after a free, a new allocation) and an in-place update
    both prepare again."""
    import torch

    from kernelswift_b200 import fused_moe as fm

    calls = []
    monkeypatch.setattr(fm, "prepare_weights", lambda *a, **k: calls.append(a) or object())
    monkeypatch.setattr(fm, "_prep_cache", {})
    w1, w2 = torch.zeros(2, 8, 64), torch.zeros(2, 64, 4)
    p1 = fm._cached_prepare(w1, w2, "none", torch.bfloat16, None, None)
    assert fm._cached_prepare(w1, w2, "none", torch.bfloat16, None, None) is p1
    assert len(calls) == 1
    alias = w1.view(w1.shape)  # same data_ptr, shape and version counter
    assert alias.data_ptr() == w1.data_ptr() and alias._version == w1._version
    assert fm._cached_prepare(alias, w2, "none", torch.bfloat16, None, None) is not p1
    assert len(calls) == 2
    w2.add_(1.0)
    fm._cached_prepare(alias, w2, "none", torch.bfloat16, None, None)
    assert len(calls) == 3


def test_launch_count_query_without_gpu():
    """moe_fused_experts_launches answers from the plan alone."""
    import torch

    from kernelswift_b200 import fused_moe as fm

    assert fm.fused_experts_launches(4096, 4096, 14336, 8, 2) == 7      # 3-launch align..sum
    assert fm.fused_experts_launches(1, 2048, 768, 128, 8) == 2         # decode kernels
    assert fm.fused_moe_launches(1, 2048, 768, 128, 8) == 2             # decode, routing inside
    assert fm.fused_moe_launches(1, 2048, 768, 128, 8,
                                 logits_dtype=torch.bfloat16) == 3      # routing kernel + decode
    assert fm.fused_moe_launches(1, 256, 128, 512, 8) == 3              # 512 experts: routing kernel
    assert fm.fused_moe_launches(4096, 4096, 14336, 8, 2) == 8          # routing + 7
    assert fm.fused_experts_launches(64, 2048, 768, 128, 8) == 6        # split gate-up
    assert fm.fused_experts_launches(64, 7168, 2048, 256, 8, "fp8") == 6
    assert fm.fused_experts_launches(20000, 512, 256, 8, 1) == 7        # 3-launch align
    assert fm.fused_experts_launches(16384, 4096, 14336, 4, 1, rows_only=True) == 6
    assert fm.fused_experts_launches(0, 512, 256, 8, 2) == 0
    assert fm.fused_experts_launches(1024, 4096, 14336, 8, 2) == 5      # 2048 ids: 1-launch align
    assert fm.fused_experts_launches(1025, 4096, 14336, 8, 2) == 7      # 2050 ids: 3-launch align


def test_plan_query_without_gpu():
    """moe_fused_experts_plan: tile widths divide the GEMMs' widths, fp8 keeps
    128/256-wide tiles and no gate-up split, decode shapes take the decode
    kernels."""
    from kernelswift_b200 import fused_moe as fm

    for T, H, I, E, k, quant in [(4096, 4096, 14336, 8, 2, "none"), (64, 2048, 768, 128, 8, "none"),
                                 (4096, 7168, 2048, 256, 8, "fp8"),
                                 (4096, 7168, 2048, 256, 8, "fp8-ue8m0"),
                                 (8192, 2048, 768, 128, 8, "int8")]:
        plan = fm.fused_experts_plan(T, H, I, E, k, quant)
        assert (2 * I) % plan["gate_up_block_n"] == 0 and H % plan["down_block_n"] == 0
        assert plan["gate_up_splits"] >= 1 and plan["down_splits"] >= 1
        assert plan["sms"] == 148 and plan["decode_path"] == 0
        assert plan["token_gather"] == (0 if quant == "int8" else 1)
        if quant.startswith("fp8"):
            assert plan["gate_up_splits"] == 1
            assert plan["gate_up_block_n"] in (128, 256) and plan["down_block_n"] in (128, 256)
    decode = fm.fused_experts_plan(1, 2048, 768, 128, 8)
    assert decode["decode_path"] == 1 and decode["token_gather"] == 0
    assert fm.fused_experts_plan(4096, 4096, 14336, 8, 2)["down_rows_dtype"] == _lib.DT_BF16


def test_plan_switches_in_a_child_process():
    """MOE_BLOCK_N forces the tile width it divides (fp8 keeps 128/256);
    MOE_NO_TOKEN_GATHER=1 turns the token-major gather off."""
    import json
    import subprocess
    import sys
    from pathlib import Path

    root = Path(__file__).resolve().parent.parent
    code = ("import json, sys; sys.path.insert(0, %r)\n"
            "from kernelswift_b200 import fused_moe as fm\n"
            "print(json.dumps([fm.fused_experts_plan(*a) for a in [\n"
            "  (4096, 4096, 14336, 8, 2), (512, 4096, 14336, 8, 2),\n"
            "  (4096, 7168, 2048, 256, 8, 'fp8'), (8192, 2048, 768, 128, 8, 'int8')]]))\n"
            % str(root))

    def plans(**env):
        res = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                             env=dict(os.environ, **env), timeout=300)
        assert res.returncode == 0, res.stderr[-2000:]
        return json.loads(res.stdout.strip().splitlines()[-1])

    forced = plans(MOE_BLOCK_N="128")
    assert all(p["down_block_n"] == 128 and p["gate_up_block_n"] == 128 for p in forced)
    narrow = plans(MOE_BLOCK_N="64")
    assert narrow[0]["down_block_n"] == 64 and narrow[2]["down_block_n"] in (128, 256)
    assert [p["token_gather"] for p in plans()] == [1, 1, 1, 0]
    assert [p["token_gather"] for p in plans(MOE_NO_TOKEN_GATHER="1")] == [0, 0, 0, 0]


def test_ep_plan_workspace_query_without_gpu():
    lib = _lib.load()
    n = ctypes.c_size_t(123)
    assert lib.moe_ep_plan_workspace_size(8192, 8, ctypes.byref(n)) == 0 and n.value == 0
    assert lib.moe_ep_plan_workspace_size(8193, 8, ctypes.byref(n)) == 0
    assert n.value == 9 * 9 * 4  # ceil(8193 / 1024) chunks x (world + 1) buckets
    assert lib.moe_ep_plan_workspace_size(65536, 128, ctypes.byref(n)) == 0
    assert n.value == 64 * 129 * 4
    assert lib.moe_ep_plan_workspace_size(100, 129, ctypes.byref(n)) == _lib.MOE_ERR_UNSUPPORTED
