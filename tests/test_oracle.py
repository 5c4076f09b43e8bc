"""CPU tests: the oracle against the reference's own outputs (tests/golden)."""
import numpy as np
import pytest
import torch

from cases import CASES, GROUPED_CASES, digest, make_grouped_inputs, make_inputs
from oracle import moe_oracle as orc

GOLDEN = __import__("pathlib").Path(__file__).resolve().parent / "golden"


def load(c):
    return np.load(GOLDEN / f"{c.name}.npz")


@pytest.mark.parametrize("case", CASES, ids=lambda c: c.name)
def test_inputs_regenerate(case):
    hidden, logits, w1, w2 = make_inputs(case)
    assert str(load(case)["digest"]) == digest(hidden, logits, w1, w2)


@pytest.mark.parametrize("case", CASES, ids=lambda c: c.name)
def test_routing_ids_match_reference(case):
    _, logits, _, _ = make_inputs(case)
    _, ids = orc.route(logits, case.k, case.renormalize)
    assert torch.equal(ids.to(torch.int32), torch.from_numpy(load(case)["topk_ids"]))


@pytest.mark.parametrize("case", CASES, ids=lambda c: c.name)
def test_forward_matches_reference(case):
    """fp32 oracle vs base.py. fp32 cases agree to fp32 rounding; bf16/fp16
    cases differ by the reference's own low-precision roundings and are held
    to the operator tolerance (rtol 2e-2, atol 2e-2)."""
    hidden, logits, w1, w2 = make_inputs(case)
    out, _, _ = orc.model_forward(hidden, logits, w1, w2, case.k, case.renormalize)
    ref = torch.from_numpy(load(case)["out"])
    if case.dtype == torch.float32:
        torch.testing.assert_close(out, ref, rtol=1e-4, atol=1e-5)
    else:
        torch.testing.assert_close(out, ref, rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("case", CASES, ids=lambda c: c.name)
def test_align_matches_reference_grouping(case):
    """Per expert, the non-padding slots of the oracle's sorted ids are the
    rows base.py:65-68 gathers with `x_rep[flat_ids == e]`, in that order."""
    g = load(case)
    ids = torch.from_numpy(g["topk_ids"])
    rows, offs = g["expert_rows"], g["expert_offsets"]
    for bm in (16, 64, 128):
        sorted_ids, expert_ids, npp = orc.moe_align(ids, case.E, bm)
        numel = ids.numel()
        pos = 0
        for e in range(case.E):
            want = rows[offs[e]:offs[e + 1]]
            cnt = want.size
            padded = -(-cnt // bm) * bm
            assert np.array_equal(sorted_ids[pos:pos + cnt], want)
            assert np.all(sorted_ids[pos + cnt:pos + padded] == numel)
            assert np.all(expert_ids[pos // bm:(pos + padded) // bm] == e)
            pos += padded
        assert npp == pos
        assert np.all(sorted_ids[pos:] == numel)
        assert np.all(expert_ids[pos // bm:] == -1)
        assert sorted_ids.size == orc.align_buffer_len(numel, case.E, bm)


def test_align_edge_cases():
    # empty input
    s, e, n = orc.moe_align(np.zeros(0, dtype=np.int64), 4, 16)
    assert n == 0 and np.all(s == 0) and np.all(e == -1)
    # all rows to one expert, more experts than rows, dropped ids
    ids = np.array([3, 3, 3, -1, 7, 99], dtype=np.int64)
    s, e, n = orc.moe_align(ids, 8, 4)
    assert n == 8
    assert list(s[:4]) == [0, 1, 2, 6] and list(s[4:8]) == [4, 6, 6, 6]
    assert list(e[:2]) == [3, 7] and np.all(e[2:] == -1)


def test_regroup_layout():
    w1 = torch.arange(2 * 64 * 3, dtype=torch.float32).reshape(1, 128, 3) * 0 + \
        torch.arange(128, dtype=torch.float32).reshape(1, 128, 1)
    r = orc.regroup_w13(w1)[0, :, 0].long().tolist()
    assert r[:16] == list(range(0, 16)) and r[16:32] == list(range(64, 80))
    assert r[32:48] == list(range(16, 32)) and r[48:64] == list(range(80, 96))


def test_fp8_block_quant_roundtrip():
    g = torch.Generator().manual_seed(0)
    w = torch.randn(2, 256, 384, generator=g)
    q, s = orc.quant_fp8_block(w)
    assert q.dtype == torch.float8_e4m3fn and s.shape == (2, 2, 3)
    err = orc.rel_l2(orc.dequant_fp8_block(q, s), w)
    assert err < 0.04  # e4m3 has 3 mantissa bits
    assert float(q.float().abs().max()) <= 448.0


def test_int8_rows_roundtrip():
    g = torch.Generator().manual_seed(0)
    w = torch.randn(64, 512, generator=g)
    q, s = orc.quant_int8_rows(w)
    assert q.dtype == torch.int8 and s.shape == (64,)
    assert orc.rel_l2(orc.dequant_int8_rows(q, s), w) < 0.02
    z, zs = orc.quant_int8_rows(torch.zeros(3, 16))
    assert torch.all(z == 0) and torch.all(zs == 1)


def test_w8a8_oracles_close_to_fp32():
    """Sanity of the quantised oracles: e4m3 (3 mantissa bits) on x, w1 and
    w2 moves the result by ~6 % relative L2 from the unquantised fp32 result,
    int8 by ~1 %. (The operator tolerance, 5e-2, is measured against these
    dequantised oracles, not against the unquantised result.)"""
    c = CASES[3]  # cfg0 shape
    hidden, logits, w1, w2 = make_inputs(c)
    w, ids = orc.route(logits, c.k)
    ref = orc.fused_experts(hidden, w1, w2, w, ids)
    assert orc.rel_l2(orc.fused_experts_fp8(hidden, w1, w2, w, ids), ref) < 0.1
    assert orc.rel_l2(orc.fused_experts_int8(hidden, w1, w2, w, ids), ref) < 3e-2


@pytest.mark.parametrize("case", GROUPED_CASES, ids=lambda c: c.name)
def test_grouped_topk_matches_reference(case):
    """The grouped top-k restatement against the reference groupedtopk/base.py
    outputs (same CPU torch ops, so bit for bit)."""
    hidden, logits = make_grouped_inputs(case)
    ref = np.load(GOLDEN / f"{case.name}.npz")
    assert str(ref["digest"]) == digest(hidden, logits)
    w, ids = orc.grouped_topk(logits, case.topk, case.renormalize, case.num_expert_group,
                              case.topk_group, case.scoring_func, case.routed_scaling_factor)
    assert torch.equal(ids, torch.from_numpy(ref["topk_ids"]))
    assert torch.equal(w, torch.from_numpy(ref["topk_weights"]))


@pytest.mark.parametrize("case", CASES, ids=lambda c: c.name)
def test_native_forward_matches_reference(case):
    """model_forward_native -- base.py's forward restated op for op in the
    activation dtype, the CPU path bench.py times as the reference arm --
    gives base.py's own outputs: the same torch ops in the same order on
    the same inputs, so bit for bit."""
    hidden, logits, w1, w2 = make_inputs(case)
    out = orc.model_forward_native(hidden, logits, w1, w2, case.k, case.renormalize)
    ref = torch.from_numpy(load(case)["out"])
    assert out.dtype == case.dtype
    assert torch.equal(out.float(), ref)
