"""The reblock oracle pinned to the reference: the landmark-tree-v2 permutations, the
Hilbert metric samples and the metric factors of tests/golden/reblock_*.npz, which
make_golden.py produced by running the reference's own CPU path."""
from __future__ import annotations

import hashlib
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import oracle
from spark_h3_b200.hierarchy import build_reblock_hierarchy
from spark_h3_b200.synthetic import make_qkv

GOLDEN = Path(__file__).resolve().parent / "golden"
TREE_CASES = [
    ("remainder", 4133, 128, 16, (1, 1, 4133), "flat", 0),
    ("grid8k", 8192, 128, 16, (2, 64, 64), "flat", 1),
    ("hilbert4", 3000, 64, 4, (3, 20, 50), "hilbert_thw", 2),
    ("tiny", 130, 128, 16, (1, 2, 65), "flat", 3),
    ("two_rounds", 20000, 128, 16, (5, 40, 100), "flat", 4),
    ("fanout8", 6016, 128, 8, (4, 32, 47), "tile_t4h4w4", 5),
]


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def digest(t: torch.Tensor) -> str:
    return hashlib.sha256(bits(t).tobytes()).hexdigest()


@pytest.mark.parametrize("name,tokens,dim,children,grid,order,seed", TREE_CASES)
def test_tree_matches_reference(name, tokens, dim, children, grid, order, seed):
    z = np.load(GOLDEN / "reblock_tree.npz")
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(2, tokens, dim, generator=g).to(torch.bfloat16)
    assert digest(x) == str(z[f"{name}_digest"]), "seeded features differ from the ones the fixture used"
    hierarchy = build_reblock_hierarchy(tokens, children)
    perm, inverse = oracle.reblock_tree(bits(x), grid, hierarchy.split_budgets, order)
    assert np.array_equal(perm, z[f"{name}_perm"])
    assert np.array_equal(np.take_along_axis(inverse, perm, 1), np.broadcast_to(np.arange(tokens), perm.shape))
    rem = tokens % 64
    if rem:  # the protected remainder sits at the tail in root order
        tail = perm[:, tokens - rem:]
        root = oracle.initial_order(grid, order)
        rank = np.argsort(root)
        assert (np.diff(rank[tail], axis=1) > 0).all()


TREE_MODE_CASES = [
    # (name, tokens, children, final fanout, fanout mode, grid, initial order, seed)
    ("arb_two_rounds", 20000, 16, None, "arbitrary_fanout", (5, 40, 100), "flat", 21),
    ("arb_fanout8", 6016, 8, None, "arbitrary_fanout", (4, 32, 47), "tile_t4h4w4", 22),
    ("p2final_8_16", 6016, 8, 16, "power_of_two_arbitrary_final", (4, 32, 47), "flat", 23),
    ("arb_final12", 13000, 16, 12, "arbitrary_fanout", (1, 1, 13000), "flat", 24),
    ("arb_root3", 12352, 4, 3, "arbitrary_fanout", (2, 32, 193), "hilbert_thw", 25),
    ("arb_fanout64", 12800, 64, None, "arbitrary_fanout", (2, 80, 80), "flat", 26),
    ("arb_final24", 20160, 32, 24, "arbitrary_fanout", (5, 63, 64), "flat", 27),
]


@pytest.mark.parametrize("name,tokens,children,final_fanout,mode,grid,order,seed", TREE_MODE_CASES)
def test_tree_fanout_modes_match_reference(name, tokens, children, final_fanout, mode, grid, order, seed):
    """The arbitrary and power-of-two-arbitrary-final fanout modes: nodes split into 3 to 50
    children over the breadth-first split topology; the reference's own
    CPU tree (recursive_landmark_tree_v2_reference) gave the permutations."""
    import json

    z = np.load(GOLDEN / "reblock_tree_modes.npz")
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(2, tokens, 128, generator=g).to(torch.bfloat16)
    assert digest(x) == str(z[f"{name}_digest"]), "seeded features differ from the ones the fixture used"
    hierarchy = build_reblock_hierarchy(tokens, children, final_fanout=final_fanout, fanout_mode=mode)
    assert [[list(b) for _, b in rnd] for rnd in hierarchy.split_budgets] == json.loads(str(z[f"{name}_budgets"]))
    perm, inverse = oracle.reblock_tree(bits(x), grid, hierarchy.split_budgets, order)
    assert np.array_equal(perm, z[f"{name}_perm"])
    assert np.array_equal(np.take_along_axis(inverse, perm, 1), np.broadcast_to(np.arange(tokens), perm.shape))


TREE_PROXY_CASES = [
    # (name, tokens, children, fanout mode, grid, proxy_iterations, seed_rule, seed)
    ("iter0_endpoint", 4096, 4, "power_of_two_fanout", (1, 64, 64), 0, "endpoint_order", 31),
    ("iter1_farthest", 8192, 16, "power_of_two_fanout", (2, 64, 64), 1, "farthest_pair", 32),
    ("iter4_farthest", 6016, 8, "power_of_two_fanout", (4, 32, 47), 4, "farthest_pair", 33),
    ("iter1_endpoint", 4133, 16, "power_of_two_fanout", (1, 1, 4133), 1, "endpoint_order", 34),
    ("iter0_arbitrary", 6016, 8, "arbitrary_fanout", (4, 32, 47), 0, "farthest_pair", 35),
    ("iter4_endpoint_arbitrary", 20000, 16, "arbitrary_fanout", (5, 40, 100), 4, "endpoint_order", 36),
]


@pytest.mark.parametrize("name,tokens,children,mode,grid,iterations,seed_rule,seed", TREE_PROXY_CASES)
def test_tree_proxy_controls_match_reference(name, tokens, children, mode, grid, iterations, seed_rule, seed):
    """Proxy controls (landmark_v2_terminal.py:43-148): 0, 1 or 4 mean updates and
    endpoint-order seeds; the reference's own CPU tree gave the permutations."""
    z = np.load(GOLDEN / "reblock_tree_proxy.npz")
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(2, tokens, 128, generator=g).to(torch.bfloat16)
    assert digest(x) == str(z[f"{name}_digest"]), "seeded features differ from the ones the fixture used"
    hierarchy = build_reblock_hierarchy(tokens, children, fanout_mode=mode)
    perm, _ = oracle.reblock_tree(bits(x), grid, hierarchy.split_budgets, proxy_iterations=iterations,
                                  seed_rule=seed_rule)
    assert np.array_equal(perm, z[f"{name}_perm"])


TREE_FROZEN_CASES = [
    # (name, tokens, children, grid, initial order, seed)
    ("frozen_remainder", 4133, 16, (1, 1, 4133), "flat", 41),
    ("frozen_two", 130, 16, (1, 2, 65), "flat", 42),
    ("frozen_hilbert", 20000, 16, (5, 40, 100), "hilbert_thw", 43),
]


@pytest.mark.parametrize("name,tokens,children,grid,order,seed", TREE_FROZEN_CASES)
def test_tree_frozen_remainder_matches_reference(name, tokens, children, grid, order, seed):
    """A caller-chosen protected remainder (excluded_indices): the ids form the tail in root
    order, whatever their norms, and the tree splits the rest as the reference does."""
    z = np.load(GOLDEN / "reblock_tree_frozen.npz")
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(2, tokens, 128, generator=g).to(torch.bfloat16)
    assert digest(x) == str(z[f"{name}_digest"]), "seeded features differ from the ones the fixture used"
    excluded = z[f"{name}_excluded"]
    perm, _ = oracle.reblock_tree(bits(x), grid, build_reblock_hierarchy(tokens, children).split_budgets, order,
                                  excluded=excluded)
    assert np.array_equal(perm, z[f"{name}_perm"])
    tail = perm[:, tokens - tokens % 64:]
    assert (np.sort(tail, 1) == np.sort(excluded, 1)).all()


def test_qk_reblock_matches_reference():
    z = np.load(GOLDEN / "reblock_qk.npz")
    grid = tuple(int(g) for g in z["grid"])
    heads = int(z["heads"])
    T = int(np.prod(grid))
    q, k, _ = make_qkv(grid, heads, 128, seed=7, dtype=torch.bfloat16, clustered=True)
    assert digest(q) == str(z["q_digest"]) and digest(k) == str(z["k_digest"])
    samples = oracle.hilbert_midpoint_samples(grid, T // 64)
    assert np.array_equal(samples, z["samples"])
    assert np.array_equal(oracle.hilbert_midpoint_samples((61, 48, 84), 245952 // 64), z["samples_big"])
    # the tree on the reference's own features reproduces its permutations exactly
    hierarchy = build_reblock_hierarchy(T, 16)
    perm, inverse = oracle.reblock_tree(z["features"], grid, hierarchy.split_budgets)
    ref = np.concatenate([z["k_perm"].reshape(heads, T), z["q_perm"].reshape(heads, T)])
    ref_inv = np.concatenate([z["k_inv"].reshape(heads, T), z["q_inv"].reshape(heads, T)])
    assert np.array_equal(perm, ref) and np.array_equal(inverse, ref_inv)
    # metric factors (float64 here, fp32 Cholesky in the reference) and the bf16 features
    tq = oracle.Tensor(bits(q), "bfloat16")
    tk = oracle.Tensor(bits(k), "bfloat16")
    factors = oracle.metric_factors(tq, tk, samples, T)
    assert np.abs(factors - z["factors"]).max() <= 1e-4 * np.abs(z["factors"]).max()
    features = oracle.bf16_bits_to_f32(oracle.reblock_features(tq, tk, factors, T))
    ref_features = oracle.bf16_bits_to_f32(z["features"])
    assert np.abs(features - ref_features).max() <= 2 ** -7 * np.abs(ref_features).max()


M2_CASES = [
    # (name, grid, heads, m2_side, layout_reuse, seed)
    ("none_even", (2, 16, 40), 2, "none", "independent", 7),
    ("none_rem", (2, 16, 41), 2, "none", "independent", 8),
    ("key_rem", (2, 16, 41), 2, "key", "independent", 9),
    ("query_rem", (2, 16, 41), 2, "query", "independent", 10),
    ("shared_none_rem", (2, 16, 41), 2, "none", "q_from_k", 11),
]


@pytest.mark.parametrize("name,grid,heads,m2_side,reuse,seed", M2_CASES)
def test_m2_ablation_raw_sides_match_reference(name, grid, heads, m2_side, reuse, seed):
    """landmark_tree_v2_m2_side (spark_integration.py:450-693): a side without the M2 factor
    clusters its raw rows, with the protected tail the baseline (both-side) features choose.
    The raw sides' permutations equal the reference's own; the factored sides go through the
    factors, whose fp32 order is a library internal (pinned separately, given the factors)."""
    z = np.load(GOLDEN / "reblock_m2.npz")
    q, k, _ = make_qkv(grid, heads, 128, seed=seed, dtype=torch.bfloat16, clustered=True)
    assert digest(q) == str(z[f"{name}_q_digest"]) and digest(k) == str(z[f"{name}_k_digest"])
    T = int(np.prod(grid))
    raw_k = bits(k[0].permute(1, 0, 2).contiguous())  # [H, T, 128]
    raw_q = bits(q[0].permute(1, 0, 2).contiguous())
    tq, tk = oracle.Tensor(bits(q), "bfloat16"), oracle.Tensor(bits(k), "bfloat16")
    samples = oracle.hilbert_midpoint_samples(grid, T // 64)
    features = oracle.reblock_features(tq, tk, oracle.metric_factors(tq, tk, samples, T), T)
    excluded = oracle.remainder_ids(features) if T % 64 else None
    budgets = build_reblock_hierarchy(T, 16).split_budgets
    if reuse == "q_from_k":
        perm, _ = oracle.reblock_tree(raw_k, grid, budgets, excluded=None if excluded is None else excluded[:heads])
        assert np.array_equal(perm, z[f"{name}_k_perm"].reshape(heads, T))
        assert np.array_equal(perm, z[f"{name}_q_perm"].reshape(heads, T))
        return
    if m2_side in ("query", "none"):
        perm, _ = oracle.reblock_tree(raw_k, grid, budgets, excluded=None if excluded is None else excluded[:heads])
        assert np.array_equal(perm, z[f"{name}_k_perm"].reshape(heads, T))
    if m2_side in ("key", "none"):
        perm, _ = oracle.reblock_tree(raw_q, grid, budgets, excluded=None if excluded is None else excluded[heads:])
        assert np.array_equal(perm, z[f"{name}_q_perm"].reshape(heads, T))
