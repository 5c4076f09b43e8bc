"""CPU: the index arithmetic of the grouped GEMM's opt-in variants, restated
and exercised before they run on a GPU.

Tail split (TAIL): over many tile counts the work items cover every (tile,
k-block) once, tail items land on distinct CTAs within the grid's last
pass, workspace slots stay inside the gridDim.x slots and are unique, no
part is empty, and adding the parts in part order equals the whole-tile sum.
Half tiles (HALF): the half-empty test of an m-block agrees with align's
layout."""
import random

import pytest


def tail_split(total_tiles, grid, k_blocks, splits=1, have_ws=True):
    """(tail_start, parts, per_part) as every CTA of the kernel derives them."""
    tail_start, parts, per_part = total_tiles, 1, 0
    R = total_tiles % grid
    if have_ws and splits == 1 and R > 0:
        f = min(grid // R, k_blocks)
        if f >= 2:
            per_part = (k_blocks + f - 1) // f
            fe = (k_blocks + per_part - 1) // per_part
            if fe >= 2:
                parts, tail_start = fe, total_tiles - R
    return tail_start, parts, per_part


def item(i, tail_start, parts, per_part, k_blocks):
    """item i -> (tile, kb0, kb1, part); part -1 = a whole tile."""
    if i >= tail_start:
        j, part = divmod(i - tail_start, parts)
        kb0 = part * per_part
        return tail_start + j, kb0, min(kb0 + per_part, k_blocks), part
    return i, 0, k_blocks, -1


CASES = [(t, g, kb) for t in (1, 5, 36, 72, 100, 147, 148, 149, 168, 184, 296, 1072, 4160)
         for g in (148, 132) for kb in (1, 3, 8, 16, 56, 224)]


@pytest.mark.parametrize("total_tiles,grid,k_blocks", CASES)
def test_items_cover_each_tile_k_block_once(total_tiles, grid, k_blocks):
    tail_start, parts, per_part = tail_split(total_tiles, grid, k_blocks)
    total_items = tail_start + (total_tiles - tail_start) * parts
    covered = {}
    per_cta = {}
    slots = set()
    for i in range(total_items):
        tile, kb0, kb1, part = item(i, tail_start, parts, per_part, k_blocks)
        assert 0 <= tile < total_tiles
        assert 0 <= kb0 < kb1 <= k_blocks, "empty or out-of-range part"
        for kb in range(kb0, kb1):
            assert (tile, kb) not in covered
            covered[(tile, kb)] = part
        cta = i % grid
        per_cta.setdefault(cta, []).append(part)
        if part >= 0:
            j = tile - tail_start
            slot = j * parts + part
            assert 0 <= slot < grid, "workspace slot beyond gridDim.x"
            assert slot not in slots
            slots.add(slot)
    assert len(covered) == total_tiles * k_blocks
    # every CTA runs the whole-tile passes, then at most one tail item
    for parts_seen in per_cta.values():
        assert sum(1 for q in parts_seen if q >= 0) <= 1
    if parts > 1:
        assert (total_tiles - tail_start) * parts <= grid
        assert total_tiles - tail_start == total_tiles % grid


def test_split_engages_only_without_k_split_and_with_workspace():
    assert tail_split(168, 148, 56)[1] > 1
    assert tail_split(168, 148, 56, splits=2)[1] == 1
    assert tail_split(168, 148, 56, have_ws=False)[1] == 1
    assert tail_split(296, 148, 56)[1] == 1      # whole waves: nothing to split
    assert tail_split(147, 148, 56)[1] == 1      # 147 tail tiles: 148 // 147 = 1


def test_part_order_sum_equals_whole_tile_sum():
    """The last part to arrive adds the parts in part order 0..parts-1, so
    the sum of a tile is the same whichever CTA finishes last; with int32
    words (kind::i8) it equals the single-accumulator sum exactly."""
    rng = random.Random(0)
    k_blocks = 224
    tail_start, parts, per_part = tail_split(1072, 148, k_blocks)
    assert parts == 4
    per_kb = [rng.randint(-2 ** 20, 2 ** 20) for _ in range(k_blocks)]
    partials = [sum(per_kb[q * per_part:min((q + 1) * per_part, k_blocks)])
                for q in range(parts)]
    for arrival in ([0, 1, 2, 3], [3, 1, 0, 2], [2, 3, 1, 0]):
        count = 0
        for q in arrival:
            count += 1
            if count == parts:  # this part finishes the tile
                total = 0
                for q2 in range(parts):
                    total += partials[q2]
                assert total == sum(per_kb)


def test_half_tile_rule_matches_align_layout():
    """The M = 64 variant treats an m-block as half-empty when its row 64 is
    the padding sentinel. That is exact because align packs an expert's rows
    at the front of its blocks: in every block the valid rows form a prefix,
    so a sentinel at row 64 means rows 64..127 are all padding, and the
    valid rows (< 64) are the rows an M = 64 MMA computes."""
    import torch

    from oracle import moe_oracle as orc

    g = torch.Generator().manual_seed(3)
    for T, E, k in [(37, 8, 2), (300, 16, 4), (1000, 64, 8), (5, 128, 8)]:
        _, ids = orc.route(torch.randn(T, E, generator=g), k)
        sorted_ids, expert_ids, npp = orc.moe_align(ids, E, 128)
        numel = T * k
        s = torch.as_tensor(sorted_ids)
        for b in range(int(npp) // 128):
            blk = s[b * 128:(b + 1) * 128]
            valid = blk < numel
            n = int(valid.sum())
            assert n > 0 and bool(valid[:n].all()), "valid rows are not a prefix"
            assert (int(blk[64]) >= numel) == (n <= 64)
