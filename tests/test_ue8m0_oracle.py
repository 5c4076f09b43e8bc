"""CPU: the fp8 path with power-of-two (UE8M0) block scales -- the oracle's
exponent rule, quantisers and scale-factor image layout, and the library's
image-size query (a host function, no GPU needed)."""
import math

import pytest
import torch

from kernelswift_b200 import _lib
from oracle import moe_oracle as orc


def test_byte_rule_is_smallest_power_of_two():
    g = torch.Generator().manual_seed(0)
    mags = torch.pow(10.0, torch.empty(20000).uniform_(-30, 30, generator=g))
    edges = torch.tensor([448.0 * 2.0 ** k for k in range(-100, 100)])
    nudged = torch.cat([edges, torch.nextafter(edges, torch.full_like(edges, math.inf)),
                        torch.nextafter(edges, torch.zeros_like(edges))])
    amax = torch.cat([mags, nudged]).float()
    b = orc.ue8m0_byte(amax)
    for a, bb in zip(amax.tolist(), b.tolist()):
        s = 2.0 ** (bb - 127)
        assert a <= 448.0 * s, (a, bb)
        assert a > 448.0 * s / 2, (a, bb)  # minimal (normal amax)


def test_byte_rule_edge_groups():
    b = orc.ue8m0_byte(torch.tensor([0.0, -0.0, 1e-42, float("nan")]))
    assert b.tolist() == [127, 127, 0, 127]


def test_block_quant_uses_top_binade_and_round_trips():
    g = torch.Generator().manual_seed(1)
    w = torch.randn(3, 256, 384, generator=g) * torch.pow(
        10.0, torch.empty(3, 1, 1).uniform_(-3, 3, generator=g))
    q, b = orc.quant_fp8_block_ue8m0(w)
    assert b.shape == (3, 2, 3)
    qf = q.float().reshape(3, 2, 128, 3, 128)
    qmax = qf.abs().amax(dim=(2, 4))
    # amax / scale lies in (224, 448], so the block's largest code is at
    # least 224 (a value just above 224 rounds down to it)
    assert bool((qmax <= 448).all()) and bool((qmax >= 224).all())
    deq = orc.dequant_fp8_block_ue8m0(q, b)
    assert orc.rel_l2(deq, w) < 0.03


def test_group_quant_round_trip():
    g = torch.Generator().manual_seed(2)
    x = torch.randn(37, 512, generator=g) * 3
    x[5] = 0  # an all-zero row: scale byte 127, zeros
    q, b = orc.quant_fp8_group_ue8m0(x)
    assert b.shape == (37, 4)
    assert b[5].tolist() == [127] * 4
    assert bool((q.float()[5] == 0).all())
    assert orc.rel_l2(orc.dequant_fp8_group_ue8m0(q, b), x) < 0.03


def test_image_round_trip_and_layout():
    g = torch.Generator().manual_seed(3)
    G, R, KB = 3, 384, 6  # KB not a multiple of 4: the last chunk column is partial
    rows = torch.randint(0, 255, (G, R, KB), generator=g)
    img = orc.sf_image_encode(rows)
    assert img.numel() == orc.sf_image_bytes(G, R, KB * 128) == G * 2 * 3 * 512
    assert torch.equal(orc.sf_image_decode(img, G, R, KB), rows)
    # inverse reading of one chunk: byte o of chunk (g, q, s) is lane o // 16,
    # cell (o % 16) // 4, k-block 4q + o % 4 of matrix row 128 s + 32 cell + lane
    q_blocks, slices = 2, 3
    for gg, qq, ss in [(0, 0, 0), (1, 1, 2), (2, 0, 1)]:
        chunk = img[((gg * q_blocks + qq) * slices + ss) * 512:][:512]
        for o in range(0, 512, 7):
            lane, cell, j = o // 16, (o % 16) // 4, o % 4
            kb = 4 * qq + j
            if kb >= KB:
                assert int(chunk[o]) == 0
                continue
            assert int(chunk[o]) == int(rows[gg, 128 * ss + 32 * cell + lane, kb])


def test_image_offsets_are_a_bijection():
    G, R, KB = 2, 256, 8
    gi, ri, ki = torch.meshgrid(torch.arange(G), torch.arange(R), torch.arange(KB), indexing="ij")
    off = orc.sf_image_offset(gi, ri, ki, 2, 2).reshape(-1)
    assert off.unique().numel() == off.numel()
    assert int(off.min()) == 0 and int(off.max()) < orc.sf_image_bytes(G, R, KB * 128)


@pytest.mark.parametrize("groups,rows,cols", [(256, 4096, 7168), (256, 7168, 2048),
                                              (1, 35328, 7168), (8, 128, 128), (3, 384, 768)])
def test_library_image_size_matches_oracle(groups, rows, cols):
    assert _lib.load().moe_ue8m0_scale_bytes(groups, rows, cols) == \
        orc.sf_image_bytes(groups, rows, cols)


def test_power_of_two_scales_cost_no_accuracy():
    """Against the unquantised fp32 layer, the e4m3 roundings of weights and
    activations cost about 6% relative L2 with either scale recipe; power-of-
    two scales (amax mapped into (224, 448] instead of onto 448) add little."""
    g = torch.Generator().manual_seed(4)
    T, H, inter, E, k = 64, 256, 256, 4, 2
    hidden = torch.randn(T, H, generator=g)
    w1 = torch.randn(E, 2 * inter, H, generator=g) / H ** 0.5
    w2 = torch.randn(E, H, inter, generator=g) / inter ** 0.5
    w, ids = orc.route(torch.randn(T, E, generator=g), k)
    ref = orc.fused_experts(hidden, w1, w2, w, ids)
    pow2 = orc.rel_l2(orc.fused_experts_fp8_ue8m0(hidden, w1, w2, w, ids), ref)
    fp32 = orc.rel_l2(orc.fused_experts_fp8(hidden, w1, w2, w, ids), ref)
    assert pow2 < 0.08 and fp32 < 0.08
    assert pow2 < 1.15 * fp32


def _kernel_sfa_chunk(mb, kb, max_m_blocks):
    """moe_grouped_gemm_mx_kernel's sfa_src: chunk (kb / 4, mb) of the
    activation image ([q][row slice] with one group)."""
    return (kb >> 2) * max_m_blocks + mb


def _kernel_sfb_chunk(e, nt, kb, q_blocks, b_slices, bn):
    """... and sfb_src: chunk (e, kb / 4, nt * BN / 128) of a weight image; a
    256-wide tile takes this chunk and the next."""
    return (e * q_blocks + (kb >> 2)) * b_slices + nt * (bn // 128)


@pytest.mark.parametrize("bn", [128, 256])
@pytest.mark.parametrize("E,N,K,rows", [(3, 512, 640, 384), (2, 1024, 2048, 256)])
def test_kernel_chunk_addressing_matches_image_layout(bn, E, N, K, rows):
    """Every bulk copy of the block-scaled GEMM lands inside its image, and
    the chunk it copies holds, at the byte the MMA selects (row r % 32 / cell
    (r % 128) / 32 / byte kb % 4), exactly the scale of each row of the tile
    for that k-block."""
    KB = K // 128
    q_blocks = -(-KB // 4)
    max_m_blocks = rows // 128
    b_slices = N // 128
    a_bytes = orc.sf_image_bytes(1, rows, K)
    b_bytes = orc.sf_image_bytes(E, N, K)
    for kb in range(KB):
        for mb in range(max_m_blocks):
            c = _kernel_sfa_chunk(mb, kb, max_m_blocks)
            assert 0 <= c * 512 and (c + 1) * 512 <= a_bytes
            for r in range(mb * 128, mb * 128 + 128):
                off = orc.sf_image_offset(0, r, kb, q_blocks, max_m_blocks)
                rr = r % 128
                assert off == c * 512 + 16 * (rr % 32) + 4 * (rr // 32) + kb % 4
        for e in range(E):
            for nt in range(N // bn):
                c = _kernel_sfb_chunk(e, nt, kb, q_blocks, b_slices, bn)
                assert (c + bn // 128) * 512 <= b_bytes
                for n in range(nt * bn, nt * bn + bn):
                    off = orc.sf_image_offset(e, n, kb, q_blocks, b_slices)
                    j, nn = divmod(n - nt * bn, 128)  # which of the tile's chunks
                    assert off == (c + j) * 512 + 16 * (nn % 32) + 4 * (nn // 32) + kb % 4
