"""Property-based tests of the host logic and the oracle's integer parts (hypothesis, CPU):
the packed layout's permutation, the Top-K / packed-route invariants with heavy ties, the
sparse query prefix and the reblock hierarchy's frontiers.  The golden fixtures pin specific
cases against the reference; these check the invariants across many generated ones."""
import math

import numpy as np
import pytest
import torch
from hypothesis import HealthCheck, given, settings
from hypothesis import strategies as st

from oracle import oracle
from spark_h3_b200 import ops
from spark_h3_b200.hierarchy import build_reblock_hierarchy
from spark_h3_b200.layout import packed_layout

SETTINGS = settings(max_examples=60, deadline=None, suppress_health_check=[HealthCheck.too_slow])


@st.composite
def tagged_sequences(draw):
    """A (t, h, w) video grid shuffled into a sequence with context rows interleaved."""
    grid = (draw(st.integers(1, 4)), draw(st.integers(1, 5)), draw(st.integers(1, 6)))
    video = [(t, h, w) for t in range(grid[0]) for h in range(grid[1]) for w in range(grid[2])]
    n_ctx = draw(st.integers(0, 12))
    seed = draw(st.integers(0, 2**31 - 1))
    rng = np.random.default_rng(seed)
    rows = [(0, p) for p in video] + [(int(rng.integers(1, 4)), tuple(int(x) for x in rng.integers(0, 7, 3)))
                                      for _ in range(n_ctx)]
    order = rng.permutation(len(rows))
    rows = [rows[i] for i in order]
    tags = torch.tensor([r[0] for r in rows], dtype=torch.long)
    pos = torch.tensor([r[1] for r in rows], dtype=torch.long)
    return tags, pos, grid


@SETTINGS
@given(tagged_sequences())
def test_packed_layout_puts_the_video_grid_first_in_raster_order(case):
    tags, pos, grid = case
    layout = packed_layout(tags, pos)
    n = tags.numel()
    perm, inv = layout.permutation, layout.inverse_permutation
    assert torch.equal(torch.sort(perm).values, torch.arange(n))
    assert torch.equal(inv[perm], torch.arange(n))
    assert layout.video_tokens == math.prod(grid) and layout.grid == grid
    head = perm[:layout.video_tokens]
    assert bool((tags[head] == 0).all())
    p = pos[head]
    keys = (p[:, 0] * grid[1] + p[:, 1]) * grid[2] + p[:, 2]
    assert torch.equal(keys, torch.arange(layout.video_tokens))  # (t, h, w) raster, each cell once
    tail = perm[layout.video_tokens:]
    assert bool((tags[tail] != 0).all()) and bool((tail[1:] > tail[:-1]).all())  # context keeps its order


@SETTINGS
@given(tagged_sequences(), st.data())
def test_packed_layout_with_one_video_row_removed(case, data):
    tags, pos, grid = case
    video_rows = torch.nonzero(tags == 0).flatten()
    if video_rows.numel() < 2:
        return
    drop = video_rows[data.draw(st.integers(0, video_rows.numel() - 1))]
    keep = torch.ones(tags.numel(), dtype=torch.bool)
    keep[drop] = False
    tags2, pos2 = tags[keep], pos[keep]
    # A missing cell leaves the grid spanned by the remaining coordinates unfilled and is
    # rejected, unless the removal dropped a whole edge row / column / plane: then the grid
    # shrinks and stays dense.
    try:
        layout = packed_layout(tags2, pos2)
    except ValueError as err:
        assert "dense grid" in str(err)
        return
    assert layout.video_tokens == math.prod(layout.grid) == video_rows.numel() - 1


@SETTINGS
@given(st.integers(1, 4), st.integers(2, 40), st.integers(0, 5), st.integers(0, 2**31 - 1))
def test_topk_route_invariants_with_ties(rows, candidates, levels, seed):
    rng = np.random.default_rng(seed)
    # Few distinct values: most rows have equal scores straddling the cut.
    scores = rng.integers(0, levels + 1, size=(1, rows, 1, candidates)).astype(np.float32)
    total = candidates + int(rng.integers(0, 40))  # blocks past the candidates are never routed
    k = int(rng.integers(1, candidates + 1))
    idx, packed = oracle.topk(scores, k, total)
    words = -(-total // 32)
    assert idx.shape == (1, rows, 1, k) and packed.shape == (1, rows, 1, words)
    for r in range(rows):
        sel = idx[0, r, 0]
        s = scores[0, r, 0]
        assert (np.diff(sel) > 0).all() and sel.min() >= 0 and sel.max() < candidates
        bits = np.unpackbits(packed[0, r, 0].view(np.uint8), bitorder="little")[:words * 32]
        assert np.array_equal(np.flatnonzero(bits), sel)
        chosen = np.zeros(candidates, dtype=bool)
        chosen[sel] = True
        if (~chosen).any():
            assert s[chosen].min() >= s[~chosen].max()
            cut = s[chosen].min()
            tied = np.flatnonzero(s == cut)
            # among equal scores at the cut, the lowest block ids are taken
            assert np.array_equal(np.sort(sel[s[sel] == cut]), tied[:int((s[sel] == cut).sum())])


@SETTINGS
@given(st.integers(1, 5000), st.floats(0.0, 1.0))
def test_target_topk_is_bounded_and_monotone(candidates, ratio):
    k = ops.target_topk(ratio, candidates)
    assert 1 <= k <= candidates
    assert k == oracle.target_topk(ratio, candidates)
    assert ops.target_topk(min(1.0, ratio + 0.05), candidates) >= k


@SETTINGS
@given(st.integers(64, 20000), st.integers(0, 2000), st.sampled_from([64, 128]))
def test_sparse_query_prefix(video, context, block):
    total = video + context
    dense = ops.sparse_query_tokens(total, video, block, "dense")
    assert dense % block == 0 and dense <= video < dense + block
    padded = math.ceil(video / block) * block
    if padded <= total:
        pad = ops.sparse_query_tokens(total, video, block, "pad")
        assert pad == padded and pad % block == 0 and pad >= video
    else:
        with pytest.raises(ValueError, match="too short to pad"):
            ops.sparse_query_tokens(total, video, block, "pad")


@SETTINGS
@given(st.integers(1, 3000), st.sampled_from([2, 4, 8, 16, 32]))
def test_reblock_hierarchy_frontiers_partition_the_leaves(blocks, children):
    h = build_reblock_hierarchy(blocks * 64, (children,))
    leaves = blocks
    for level in h.levels:
        # each frontier is a sorted partition of [0, leaves) into contiguous intervals
        assert level[0][0] == 0 and level[-1][1] == leaves
        assert all(a < b for a, b in level)
        assert all(level[i][1] == level[i + 1][0] for i in range(len(level) - 1))
    assert [tuple(x) for x in h.levels[-1]] == [(i, i + 1) for i in range(leaves)]  # 64-token leaves
    for parents, kids in zip(h.levels, h.levels[1:]):
        for a, b in parents:
            inside = [(x, y) for x, y in kids if a <= x and y <= b]
            assert sum(y - x for x, y in inside) == b - a
            assert len(inside) <= children  # no split has more children than the fanout


@settings(max_examples=25, deadline=None, suppress_health_check=[HealthCheck.too_slow])
@given(st.integers(2, 90), st.integers(0, 63), st.sampled_from([2, 4, 8, 16, 32, 64]),
       st.sampled_from([None, 3, 5, 7, 12, 24, 32]), st.sampled_from(["arbitrary_fanout",
                                                                   "power_of_two_arbitrary_final"]),
       st.integers(0, 2**31 - 1))
def test_arbitrary_fanout_trees_are_exact_partitions(blocks, rem, children, final_fanout, mode, seed):
    """Any child count from 2 to 64 over the breadth-first split topology: the oracle tree is a
    permutation of the tokens, every leaf holds its 64 tokens, the remainder sits at the tail,
    and the C-ABI plan builder accepts the hierarchy with a power-of-two level width."""
    from spark_h3_b200 import _lib, reblock

    tokens = blocks * 64 + rem
    h = build_reblock_hierarchy(tokens, children, final_fanout=final_fanout, fanout_mode=mode)
    x = torch.randn(1, tokens, 128, generator=torch.Generator().manual_seed(seed)).to(torch.bfloat16)
    bits_ = x.view(torch.int16).numpy().view(np.uint16)
    perm, inverse = oracle.reblock_tree(bits_, (1, 1, tokens), h.split_budgets)
    assert np.array_equal(np.sort(perm[0]), np.arange(tokens))
    assert np.array_equal(inverse[0][perm[0]], np.arange(tokens))
    if rem:
        assert np.array_equal(perm[0, blocks * 64:], np.sort(oracle.remainder_ids(bits_)[0]))
    schedule = reblock._schedule(h)
    lib = _lib.load()
    n = lib.sb_reblock_plan(schedule.ctypes.data, len(schedule), tokens, None, 0)
    assert n > 0
    plan = np.zeros(n, dtype=np.int32)
    assert lib.sb_reblock_plan(schedule.ctypes.data, len(schedule), tokens, plan.ctypes.data, n) == n
    for level in range(plan[0]):
        P = plan[8 + 8 * level + 3]
        assert P >= 2 and P & (P - 1) == 0 and P <= 64
