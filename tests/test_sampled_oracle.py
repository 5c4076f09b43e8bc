"""CPU: the sampled-token oracle used by the large GPU parity cases equals
the whole-batch oracle on the sampled rows, for every quantisation, and the
token picker covers every hit expert."""
import pytest
import torch

from oracle import moe_oracle as orc
from sampled import ORACLES, cover_tokens, oracle_on_tokens


@pytest.mark.parametrize("quant", sorted(ORACLES))
def test_chunked_oracle_equals_full_oracle(quant):
    T, H, I, E, k = 40, 256, 128, 16, 4
    g = torch.Generator().manual_seed(11)
    hidden = torch.randn(T, H, generator=g).to(torch.bfloat16)
    w, ids = orc.route(torch.randn(T, E, generator=g), k)
    ids[3, 1] = -1  # a dropped slot
    w1 = torch.randn(E, 2 * I, H, generator=g) / H ** 0.5
    w2 = torch.randn(E, H, I, generator=g) / I ** 0.5
    full = ORACLES[quant](hidden, w1, w2, w, ids)
    tokens = cover_tokens(ids, extra=5, seed=1)
    part = oracle_on_tokens(quant, hidden, w1, w2, w, ids, tokens, chunk=3)
    torch.testing.assert_close(part, full[tokens], rtol=1e-5, atol=1e-5)


def test_cover_tokens_hits_every_expert():
    g = torch.Generator().manual_seed(2)
    _, ids = orc.route(torch.randn(500, 64, generator=g), 8)
    tokens = cover_tokens(ids, extra=10)
    assert set(ids[tokens].unique().tolist()) == set(ids.unique().tolist())
    assert torch.equal(tokens, tokens.unique())
    assert 10 <= tokens.numel() <= 64 + 10
