"""GPU: the full operator against the reference outputs (tests/golden) and
the fp32 oracle, through the drop-in ModelNew and the functional API."""
import numpy as np
import pytest
import torch

from cases import CASES, make_inputs
from kernelswift_b200 import fused_moe as fm
from oracle import moe_oracle as orc
from sampled import cover_tokens, oracle_on_tokens

pytestmark = pytest.mark.gpu

GOLDEN = __import__("pathlib").Path(__file__).resolve().parent / "golden"
TOL = dict(rtol=2e-2, atol=2e-2)  # bf16/fp16 operands, fp32 accumulation


def auto_bench_flow(case, device):
    """What auto_bench.compare_case does (auto_bench.py:637-654): build on
    CPU, copy the reference's state_dict, move to the device, forward."""
    hidden, logits, w1, w2 = make_inputs(case)
    model = fm.ModelNew(case.E, case.k, case.H, case.I, case.renormalize)
    model.load_state_dict({"w1": w1, "w2": w2})
    model = model.to(device).eval()
    with torch.no_grad():
        out = model(hidden.to(device), logits.to(device))
    return out, (hidden, logits, w1, w2)


@pytest.mark.parametrize("case", CASES, ids=lambda c: c.name)
def test_modelnew_matches_reference_golden(cuda_device, case):
    out, (hidden, logits, w1, w2) = auto_bench_flow(case, cuda_device)
    assert out.dtype == case.dtype and out.shape == (case.T, case.H)
    ref = torch.from_numpy(np.load(GOLDEN / f"{case.name}.npz")["out"])
    # auto_bench's own criterion (auto_bench.py:313, atol=rtol=1e-2)
    torch.testing.assert_close(out.float().cpu(), ref, rtol=1e-2, atol=1e-2)
    # and the operator tolerance against the fp32 oracle
    oracle_out, _, _ = orc.model_forward(hidden, logits, w1, w2, case.k, case.renormalize)
    torch.testing.assert_close(out.float().cpu(), oracle_out, **TOL)


@pytest.mark.parametrize("name", ["toy_fp32", "cfg0_fp32", "dsv3_mini_fp32", "norenorm_fp32"])
def test_fp32_activations_compute_in_tf32(cuda_device, name):
    """fp32 activations keep fp32 operands (tf32 tensor-core GEMMs on operands
    rounded to tf32, fp32 weights prepared once): the output is within 1e-3
    relative L2 of base.py's own fp32 output (measured 5.2e-4; bf16 operands
    gave 4.1e-3)."""
    from cases import BY_NAME
    case = BY_NAME[name]
    out, _ = auto_bench_flow(case, cuda_device)
    ref = torch.from_numpy(np.load(GOLDEN / f"{name}.npz")["out"])
    assert out.dtype == torch.float32
    assert orc.rel_l2(out.cpu(), ref) <= 1e-3, orc.rel_l2(out.cpu(), ref)
    assert fm.compute_dtype_for(torch.float32) == torch.float32


def test_state_dict_is_reference_compatible():
    m = fm.ModelNew(8, 2, 128, 64)
    assert set(m.state_dict()) == {"w1", "w2"}
    assert m.w1.shape == (8, 128, 128) and m.w2.shape == (8, 128, 64)


def test_weight_update_invalidates_prepared_cache(cuda_device):
    case = CASES[0]
    hidden, logits, w1, w2 = make_inputs(case)
    m = fm.ModelNew(case.E, case.k, case.H, case.I).to(cuda_device)
    with torch.no_grad():
        m.w1.copy_(w1)
        m.w2.copy_(w2)
        a = m(hidden.to(cuda_device), logits.to(cuda_device)).clone()
        m.w2.mul_(2.0)
        b = m(hidden.to(cuda_device), logits.to(cuda_device))
    torch.testing.assert_close(b, 2 * a, rtol=1e-5, atol=1e-6)


def random_problem(T, H, I, E, k, dtype, seed, bias=0.0, device="cuda"):
    g = torch.Generator().manual_seed(seed)
    hidden = torch.randn(T, H, generator=g).to(dtype)
    logits = torch.randn(T, E, generator=g)
    if bias:
        logits = logits + torch.randn(E, generator=g) * bias
    w, ids = orc.route(logits, k)
    # weights generated on the device (large shapes), checked against a CPU
    # copy of only the experts that are hit
    gd = torch.Generator(device=device).manual_seed(seed)
    w1 = torch.randn(E, 2 * I, H, generator=gd, device=device, dtype=torch.bfloat16) / H ** 0.5
    w2 = torch.randn(E, H, I, generator=gd, device=device, dtype=torch.bfloat16) / I ** 0.5
    return hidden.to(device), w1, w2, w, ids


def oracle_subset(hidden, w1, w2, w, ids, tokens):
    """fp32 oracle on the given tokens, moving only the hit experts."""
    return oracle_on_tokens("none", hidden, w1, w2, w, ids, tokens)


# Every token/size pair of the bf16 configurations: Mixtral-8x7B (H=4096,
# I=14336, E=8, top-2) at T in {1, 16, 64, 512, 4096, 16384}, Qwen3-30B-A3B
# (H=2048, I=768, E=128, top-8, skewed routing) at T in {1, 64, 1024, 8192},
# DeepSeek-V3 (H=7168, I=2048, E=256, top-8) in bf16 at T=64 and at the
# expert-parallel configuration's 8192 tokens per GPU with all 256 experts
# on one GPU. Up to 64 tokens every token is checked; above, the first token
# of every hit expert plus `extra` random tokens.
SHAPES = [
    # name, T, H, I, E, k, logit bias std, extra random tokens
    ("mixtral_T1", 1, 4096, 14336, 8, 2, 0.0, 0),
    ("mixtral_T16", 16, 4096, 14336, 8, 2, 0.0, 0),
    ("mixtral_T64", 64, 4096, 14336, 8, 2, 0.0, 0),
    ("mixtral_T512", 512, 4096, 14336, 8, 2, 0.0, 48),
    ("mixtral_T4096", 4096, 4096, 14336, 8, 2, 0.0, 64),
    ("mixtral_T16384", 16384, 4096, 14336, 8, 2, 0.0, 64),
    ("qwen3_T1", 1, 2048, 768, 128, 8, 0.5, 0),
    ("qwen3_T64", 64, 2048, 768, 128, 8, 0.5, 0),
    ("qwen3_T1024", 1024, 2048, 768, 128, 8, 0.5, 64),
    ("qwen3_T8192", 8192, 2048, 768, 128, 8, 0.5, 128),
    ("dsv3_T64_bf16", 64, 7168, 2048, 256, 8, 0.0, 0),
    ("dsv3_T8192_bf16", 8192, 7168, 2048, 256, 8, 0.0, 64),
]


@pytest.mark.parametrize("name,T,H,I,E,k,bias,extra", SHAPES, ids=[s[0] for s in SHAPES])
def test_config_shapes_bf16(cuda_device, name, T, H, I, E, k, bias, extra):
    hidden, w1, w2, w, ids = random_problem(T, H, I, E, k, torch.bfloat16, seed=T + E,
                                            bias=bias)
    out = fm.fused_experts(hidden, w1, w2, w.to(cuda_device), ids.to(cuda_device))
    torch.cuda.synchronize()
    tokens = torch.arange(T) if T <= 64 else cover_tokens(ids, extra)
    ref = oracle_subset(hidden, w1, w2, w, ids, tokens)
    torch.testing.assert_close(out.cpu()[tokens].float(), ref, **TOL)


def test_permutation_equivariance_bit_exact(cuda_device):
    """A token's result does not depend on where it sits in the batch:
    permuting tokens permutes the output bit for bit (full Mixtral shape)."""
    T, H, I, E, k = 4096, 4096, 14336, 8, 2
    hidden, w1, w2, w, ids = random_problem(T, H, I, E, k, torch.bfloat16, seed=3)
    w, ids = w.to(cuda_device), ids.to(cuda_device)
    out = fm.fused_experts(hidden, w1, w2, w, ids).clone()
    perm = torch.randperm(T, generator=torch.Generator().manual_seed(1)).to(cuda_device)
    out_p = fm.fused_experts(hidden[perm], w1, w2, w[perm], ids[perm])
    assert torch.equal(out_p, out[perm])
    tokens = torch.randperm(T, generator=torch.Generator().manual_seed(2))[:32]
    ref = oracle_subset(hidden, w1, w2, w.cpu(), ids.cpu(), tokens)
    torch.testing.assert_close(out.cpu()[tokens].float(), ref, **TOL)


def test_deterministic(cuda_device):
    hidden, w1, w2, w, ids = random_problem(1024, 2048, 768, 128, 8, torch.bfloat16, seed=4,
                                            bias=0.5)
    w, ids = w.to(cuda_device), ids.to(cuda_device)
    a = fm.fused_experts(hidden, w1, w2, w, ids).clone()
    for _ in range(3):
        assert torch.equal(fm.fused_experts(hidden, w1, w2, w, ids), a)


def test_int32_ids_and_bf16_weights(cuda_device):
    hidden, w1, w2, w, ids = random_problem(100, 512, 256, 16, 4, torch.bfloat16, seed=6)
    a = fm.fused_experts(hidden, w1, w2, w.to(cuda_device), ids.to(cuda_device)).clone()
    b = fm.fused_experts(hidden, w1, w2, w.to(torch.bfloat16).to(cuda_device),
                         ids.to(torch.int32).to(cuda_device))
    torch.testing.assert_close(a, b, rtol=1e-2, atol=1e-2)


def test_dropped_ids_contribute_nothing(cuda_device):
    hidden, w1, w2, w, ids = random_problem(64, 512, 256, 8, 2, torch.bfloat16, seed=8)
    ids2 = ids.clone()
    ids2[::3, 1] = -1
    out = fm.fused_experts(hidden, w1, w2, w.to(cuda_device), ids2.to(cuda_device))
    ref = orc.fused_experts(hidden.cpu(), w1.cpu(), w2.cpu(), w, ids2)
    torch.testing.assert_close(out.cpu().float(), ref, **TOL)


def test_empty_batch(cuda_device):
    hidden = torch.empty(0, 128, dtype=torch.bfloat16, device=cuda_device)
    w1 = torch.randn(4, 128, 128, device=cuda_device)
    w2 = torch.randn(4, 128, 64, device=cuda_device)
    out = fm.fused_experts(hidden, w1, w2, torch.empty(0, 2, device=cuda_device),
                           torch.empty(0, 2, dtype=torch.int64, device=cuda_device))
    assert out.shape == (0, 128)


def test_rejects_cpu_tensors():
    with pytest.raises(ValueError, match="CUDA"):
        fm.fused_experts(torch.zeros(2, 128), torch.zeros(2, 128, 128), torch.zeros(2, 128, 64),
                         torch.zeros(2, 1), torch.zeros(2, 1, dtype=torch.int64))


def test_rejects_other_activation(cuda_device):
    with pytest.raises(ValueError, match="activation"):
        fm.fused_experts(torch.zeros(2, 128, device=cuda_device), None, None,
                         torch.zeros(2, 1), torch.zeros(2, 1, dtype=torch.int64),
                         activation="gelu")


def test_captured_graph_matches_eager(cuda_device):
    """CapturedMoE replays the same kernels: bit-identical to eager calls,
    also after new inputs are copied into the static buffers."""
    T, H, I, E, k = 16, 512, 256, 8, 2
    m = fm.ModelNew(E, k, H, I).to(cuda_device)
    g = torch.Generator(device=cuda_device).manual_seed(0)
    with torch.no_grad():
        m.w1.normal_(0, H ** -0.5, generator=g)
        m.w2.normal_(0, I ** -0.5, generator=g)
    cap = fm.CapturedMoE(m, T, H, E, dtype=torch.bfloat16, device=cuda_device)
    for seed in (1, 2):
        gi = torch.Generator(device=cuda_device).manual_seed(seed)
        hidden = torch.randn(T, H, generator=gi, device=cuda_device).to(torch.bfloat16)
        logits = torch.randn(T, E, generator=gi, device=cuda_device)
        with torch.no_grad():
            eager = m(hidden, logits).clone()
        out = cap(hidden, logits)
        torch.cuda.synchronize()
        assert torch.equal(out, eager)


@pytest.mark.parametrize("T", [5, 3000])
def test_rows_only_matches_full_forward(cuda_device, T):
    """moe_fused_experts_rows (top_k = 1, the expert-parallel receive buffer):
    the rows of tokens with a valid id equal moe_fused_experts' bit for bit,
    whether the down GEMM writes them directly (unsplit) or the sum does."""
    H, I, E = 256, 512, 8
    g = torch.Generator().manual_seed(T)
    hidden = torch.randn(T, H, generator=g).to(torch.bfloat16).to(cuda_device)
    w1 = (torch.randn(E, 2 * I, H, generator=g) / H ** 0.5).to(torch.bfloat16).to(cuda_device)
    w2 = (torch.randn(E, H, I, generator=g) / I ** 0.5).to(torch.bfloat16).to(cuda_device)
    ids = torch.randint(-1, E, (T, 1), generator=g, dtype=torch.int32).to(cuda_device)
    ones = torch.ones(T, 1, device=cuda_device)
    prep = fm.prepare_weights(w1, w2, "none", torch.bfloat16)
    full = fm.fused_experts(hidden, prep, None, ones, ids)
    rows = torch.full_like(hidden, float("nan"))
    fm.fused_experts(hidden, prep, None, ones, ids, out=rows, rows_only=True)
    valid = (ids.view(-1) >= 0).cpu()
    assert torch.equal(rows.cpu()[valid], full.cpu()[valid])


def test_host_pipeline_matches_direct_calls(cuda_device):
    """HostPipeline: several steps with different host inputs and outputs,
    copies overlapped across steps; each output equals a direct forward."""
    T, H, I, E, k = 64, 256, 512, 8, 2
    g = torch.Generator().manual_seed(5)
    model = fm.ModelNew(E, k, H, I).to(cuda_device)
    with torch.no_grad():
        model.w1.copy_(torch.randn(E, 2 * I, H, generator=g) / H ** 0.5)
        model.w2.copy_(torch.randn(E, H, I, generator=g) / I ** 0.5)
    cap = fm.CapturedMoE(model, T, H, E, dtype=torch.bfloat16, device=cuda_device)
    for fn in (model, cap):
        pipe = fm.HostPipeline(fn, T, H, E, dtype=torch.bfloat16, device=cuda_device)
        ins = [(torch.randn(T, H, generator=g).to(torch.bfloat16).pin_memory(),
                torch.randn(T, E, generator=g).pin_memory()) for _ in range(5)]
        outs = [torch.empty(T, H, dtype=torch.bfloat16).pin_memory() for _ in range(5)]
        for (h, l), o in zip(ins, outs):
            pipe.submit(h, l, o)
        pipe.flush()
        torch.cuda.synchronize()
        for (h, l), o in zip(ins, outs):
            with torch.no_grad():
                ref = model(h.to(cuda_device), l.to(cuda_device))
            assert torch.equal(o, ref.cpu())
