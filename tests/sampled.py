"""Test helpers: the oracle on a sample of a large batch's tokens.

At the full layer sizes the oracle cannot hold every expert on the host
(DeepSeek-V3's 256 experts are 45 GB in fp32), so these helpers evaluate it
on chosen tokens only, moving the experts those tokens hit to the host in
chunks and adding each chunk's contribution. Every quantisation the
oracles apply is per expert (weight blocks, weight rows) or per token
(activation groups), so a chunk's contribution is exactly its part of the
full oracle's sum; only the fp32 summation order over a token's slots
differs.
"""
from __future__ import annotations

import torch

from oracle import moe_oracle as orc

ORACLES = {
    "none": orc.fused_experts,
    "fp8": orc.fused_experts_fp8,
    "fp8-ue8m0": orc.fused_experts_fp8_ue8m0,
    "int8": orc.fused_experts_int8,
}


def cover_tokens(ids: torch.Tensor, extra: int, seed: int = 0) -> torch.Tensor:
    """Sorted token indices: the first token routed to each expert that any
    token hits (so every hit expert's weights are checked), plus `extra`
    random tokens."""
    ids = ids.cpu()
    T, k = ids.shape
    flat = ids.reshape(-1)
    valid = flat >= 0
    tok = torch.arange(T).repeat_interleave(k)[valid]
    ex = flat[valid]
    first = torch.full((int(ex.max()) + 1 if ex.numel() else 1,), T, dtype=torch.int64)
    first.scatter_reduce_(0, ex, tok, reduce="amin")
    chosen = first[first < T]
    rnd = torch.randperm(T, generator=torch.Generator().manual_seed(seed))[:extra]
    return torch.unique(torch.cat([chosen, rnd]))


def oracle_on_tokens(quant: str, hidden, w1, w2, w, ids, tokens, chunk: int = 16):
    """fp32 oracle output [len(tokens), H] for the given tokens; weights may
    live on the GPU, experts are moved to the host `chunk` at a time."""
    f = ORACLES[quant]
    tokens = tokens.cpu()
    x = hidden[tokens.to(hidden.device)].cpu()
    sub = ids.cpu()[tokens]
    wsub = w.cpu()[tokens].float()
    hit = torch.unique(sub[sub >= 0])
    out = torch.zeros(x.shape[0], x.shape[1], dtype=torch.float32)
    E = w1.shape[0]
    for c in range(0, hit.numel(), chunk):
        exps = hit[c:c + chunk]
        remap = torch.full((E,), -1, dtype=torch.int64)
        remap[exps] = torch.arange(exps.numel())
        sid = torch.where(sub >= 0, remap[sub.clamp(min=0)], torch.full_like(sub, -1))
        dev_idx = exps.to(w1.device)
        out += f(x, w1[dev_idx].float().cpu(), w2[dev_idx].float().cpu(), wsub, sid)
    return out
