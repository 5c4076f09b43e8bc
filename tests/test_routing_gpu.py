"""GPU: the fused routing kernel (moe_topk_softmax) against base.py's torch
routing (softmax -> topk -> renormalise, base.py:44-48), and the grouped
top-k kernel (moe_grouped_topk) against the reference groupedtopk/base.py
outputs (tests/golden/gtk_*.npz) and the oracle."""
import numpy as np
import pytest
import torch

from cases import CASES, GROUPED_CASES, make_grouped_inputs, make_inputs
from kernelswift_b200 import fused_moe as fm
from oracle import moe_oracle as orc

pytestmark = pytest.mark.gpu

GOLDEN = __import__("pathlib").Path(__file__).resolve().parent / "golden"


def torch_route(logits, k, renorm):
    scores = torch.softmax(logits.float(), dim=-1)
    w, ids = torch.topk(scores, k, dim=-1)
    if renorm:
        w = w / w.sum(-1, keepdim=True)
    return w, ids


@pytest.mark.parametrize("case", CASES, ids=lambda c: c.name)
def test_ids_match_reference_golden(cuda_device, case):
    hidden, logits, _, _ = make_inputs(case)
    w, ids = fm.fused_topk(hidden.to(cuda_device), logits.to(cuda_device), case.k,
                           case.renormalize)
    want = torch.from_numpy(np.load(GOLDEN / f"{case.name}.npz")["topk_ids"])
    assert torch.equal(ids.cpu(), want)


@pytest.mark.parametrize("T,E,k,bias,renorm", [
    (4096, 8, 2, 0.0, True),
    (8192, 128, 8, 0.5, True),
    (4096, 256, 8, 0.0, True),
    (1000, 64, 6, 1.0, False),
    (333, 1024, 8, 0.0, True),
    (1, 8, 2, 0.0, True),
    (77, 40, 32, 0.0, True),
])
def test_matches_torch_routing_fp32_logits(cuda_device, T, E, k, bias, renorm):
    """fp32 logits (no exact ties): ids bit-identical to torch.topk."""
    g = torch.Generator().manual_seed(T + E)
    logits = (torch.randn(T, E, generator=g) + torch.randn(E, generator=g) * bias).to(cuda_device)
    hidden = torch.empty(T, 8, device=cuda_device)
    w, ids = fm.fused_topk(hidden, logits, k, renorm)
    rw, rids = torch_route(logits, k, renorm)
    assert torch.equal(ids.long(), rids)
    torch.testing.assert_close(w, rw, rtol=1e-5, atol=1e-6)


def test_bf16_logits_with_exact_ties(cuda_device):
    """bf16 logits tie exactly and often; torch.topk leaves the order of tied
    values unspecified. Ours must be a valid top-k (every selected logit >=
    every unselected one), in descending order with ties to the lower index,
    and its weights equal torch's position by position (tied experts have
    equal weights)."""
    T, E, k = 2048, 128, 8
    g = torch.Generator().manual_seed(5)
    logits = (torch.randn(T, E, generator=g) + torch.randn(E, generator=g) * 0.5)
    logits = logits.to(torch.bfloat16).to(cuda_device)
    hidden = torch.empty(T, 8, device=cuda_device)
    w, ids = fm.fused_topk(hidden, logits, k, True)
    rw, rids = torch_route(logits, k, True)
    lf = logits.float()
    sel = torch.gather(lf, 1, ids.long())
    mask = torch.ones_like(lf, dtype=torch.bool)
    mask.scatter_(1, ids.long(), False)
    unsel_max = torch.where(mask, lf, torch.full_like(lf, -float("inf"))).amax(1)
    assert bool((sel.min(1).values >= unsel_max).all())
    assert bool((sel[:, :-1] >= sel[:, 1:]).all())
    tie = sel[:, :-1] == sel[:, 1:]
    assert bool((ids[:, :-1][tie] < ids[:, 1:][tie]).all())
    torch.testing.assert_close(w, rw, rtol=1e-5, atol=1e-6)
    # the tie-free rows agree with torch exactly
    no_tie = ~(sel[:, :-1] == sel[:, 1:]).any(1) & (sel[:, -1] > unsel_max)
    assert torch.equal(ids.long()[no_tie], rids[no_tie])


def test_weights_in_activation_dtype_and_int64_ids(cuda_device):
    logits = torch.randn(50, 16, device=cuda_device)
    hidden = torch.empty(50, 8, device=cuda_device)
    w, ids = fm.fused_topk(hidden, logits, 4, True, weights_dtype=torch.bfloat16,
                           ids_dtype=torch.int64)
    rw, rids = torch_route(logits, 4, True)
    assert w.dtype == torch.bfloat16 and ids.dtype == torch.int64
    assert torch.equal(ids, rids)
    torch.testing.assert_close(w, rw.to(torch.bfloat16), rtol=8e-3, atol=1e-6)


def test_ties_go_to_the_lower_expert(cuda_device):
    logits = torch.zeros(3, 8, device=cuda_device)
    logits[1, 5] = 1.0
    hidden = torch.empty(3, 8, device=cuda_device)
    _, ids = fm.fused_topk(hidden, logits, 3, True)
    assert ids.cpu().tolist() == [[0, 1, 2], [5, 0, 1], [0, 1, 2]]


# ---------------------------------------------------------------------------
# grouped top-k (kernels/track1-triton/groupedtopk/base.py)
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("case", GROUPED_CASES, ids=lambda c: c.name)
def test_grouped_topk_matches_reference_golden(cuda_device, case):
    """moe_grouped_topk against the reference operator's own outputs: ids
    bit-exact, fp32 weights to a few ulp (exp/sigmoid evaluated on the GPU)."""
    hidden, logits = make_grouped_inputs(case)
    ref = np.load(GOLDEN / f"{case.name}.npz")
    model = fm.GroupedTopK(case.topk, case.renormalize, case.num_expert_group,
                           case.topk_group, case.scoring_func, case.routed_scaling_factor)
    w, ids = model(hidden.to(cuda_device), logits.to(cuda_device))
    assert w.dtype == torch.float32 and ids.dtype == torch.int32
    assert torch.equal(ids.cpu(), torch.from_numpy(ref["topk_ids"]))
    torch.testing.assert_close(w.cpu(), torch.from_numpy(ref["topk_weights"]),
                               rtol=1e-5, atol=1e-6)


def test_grouped_topk_respects_groups_and_order(cuda_device):
    """Random problems against the oracle: every id lies in one of the
    topk_group best groups, ids are in descending score order, equal to the
    oracle's; 16-bit logits are accepted."""
    g = torch.Generator().manual_seed(3)
    for T, E, G, tg, k, sf in ((300, 128, 8, 3, 6, "sigmoid"), (1, 64, 2, 1, 4, "softmax"),
                               (129, 96, 6, 2, 5, "softmax")):
        logits = torch.randn(T, E, generator=g)
        w, ids = fm.grouped_topk(torch.empty(T, 1, device=cuda_device), logits.to(cuda_device),
                                 k, True, G, tg, sf)
        rw, rids = orc.grouped_topk(logits, k, True, G, tg, sf)
        assert torch.equal(ids.cpu(), rids)
        torch.testing.assert_close(w.cpu(), rw, rtol=1e-5, atol=1e-6)
    logits = torch.randn(40, 64, generator=g)
    for dt in (torch.bfloat16, torch.float16):
        w, ids = fm.grouped_topk(torch.empty(40, 1, device=cuda_device),
                                 logits.to(dt).to(cuda_device), 4, True, 4, 2)
        assert torch.isfinite(w).all() and ((ids >= 0) & (ids < 64)).all()


def test_grouped_topk_rejects_impossible_k(cuda_device):
    from kernelswift_b200._lib import MoeError

    logits = torch.randn(4, 32, device=cuda_device)
    with pytest.raises(MoeError):
        # 1 kept group of 8 experts cannot supply 9
        fm.grouped_topk(torch.empty(4, 1, device=cuda_device), logits, 9, True, 4, 1)
