"""Host logic of the reblock path: root orders and Hilbert metric samples against the
reference fixtures, and the node tables the C-ABI plan builder derives from the hierarchy
(no GPU needed: sb_reblock_plan is host code)."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from oracle import oracle
from spark_h3_b200 import reblock
from spark_h3_b200.hierarchy import build_reblock_hierarchy

GOLDEN = Path(__file__).resolve().parent / "golden"


def test_hilbert_samples_match_reference():
    z = np.load(GOLDEN / "reblock_qk.npz")
    grid = tuple(int(g) for g in z["grid"])
    assert np.array_equal(reblock.hilbert_midpoint_sample_indices(grid, int(np.prod(grid)) // 64), z["samples"])
    assert np.array_equal(reblock.hilbert_midpoint_sample_indices((61, 48, 84), 245952 // 64), z["samples_big"])


@pytest.mark.parametrize("order", reblock.INITIAL_ORDERS)
def test_initial_orders(order):
    grid = (3, 20, 50)
    ids = reblock.initial_token_indices(grid, order)
    assert np.array_equal(np.sort(ids), np.arange(3000))
    assert np.array_equal(ids, oracle.initial_order(grid, order))


def test_unknown_initial_order_rejected():
    with pytest.raises(ValueError, match="initial_order"):
        reblock.initial_token_indices((1, 1, 64), "spiral")


@pytest.mark.parametrize("tokens,children,final_fanout,mode", [
    (245952, 16, None, "power_of_two_fanout"), (4133, 16, None, "power_of_two_fanout"),
    (6016, 8, None, "power_of_two_fanout"), (3000, 4, None, "power_of_two_fanout"),
    (130, 16, None, "power_of_two_fanout"), (64, 16, None, "power_of_two_fanout"),
    (20000, 16, None, "arbitrary_fanout"), (13000, 16, 12, "arbitrary_fanout"),
    (6016, 8, 16, "power_of_two_arbitrary_final"), (12352, 4, 3, "arbitrary_fanout"),
    (245952, 64, None, "arbitrary_fanout")])
def test_plan_node_tables(tokens, children, final_fanout, mode):
    """Node tables of every fanout mode; a level runs with the smallest power-of-two fanout
    that holds its largest node, whatever the node's own child count."""
    from spark_h3_b200 import _lib

    h = build_reblock_hierarchy(tokens, children, final_fanout=final_fanout, fanout_mode=mode)
    schedule = reblock._schedule(h)
    lib = _lib.load()
    n = lib.sb_reblock_plan(schedule.ctypes.data, len(schedule), tokens, None, 0)
    assert n > 0
    plan = np.zeros(n, dtype=np.int32)
    assert lib.sb_reblock_plan(schedule.ctypes.data, len(schedule), tokens, plan.ctypes.data, n) == n
    levels, N, active = plan[0], plan[1], plan[2]
    assert N == tokens and active == tokens - tokens % 64
    covered_leaves = 0
    for l in range(levels):
        count, node_off, tile_off, P, S = plan[8 + 8 * l: 8 + 8 * l + 5]
        assert P >= 2 and (P & (P - 1)) == 0 and S == P - 1
        tiles = plan[tile_off: tile_off + active // 64]
        largest = max(int(plan[node_off + 68 * j + 2]) for j in range(count))
        assert P // 2 < largest <= P
        for j in range(count):
            start, size, C = plan[node_off + 68 * j: node_off + 68 * j + 3]
            caps = plan[node_off + 68 * j + 4: node_off + 68 * j + 4 + C]
            assert size == caps.sum() and (caps % 64 == 0).all() and C <= P
            assert (tiles[start // 64:(start + size) // 64] == j).all()
            covered_leaves += int((caps == 64).sum())
    assert covered_leaves == (active // 64 if active // 64 > 1 else 0)
    assert lib.sb_reblock_workspace_bytes(plan.ctypes.data, 4) > 0


def test_plan_rejects_short_schedule():
    from spark_h3_b200 import _lib

    h = build_reblock_hierarchy(4096, 16)
    schedule = reblock._schedule(h)[:3]
    assert _lib.load().sb_reblock_plan(schedule.ctypes.data, len(schedule), 4096, None, 0) < 0


def test_plan_rejects_more_than_64_children():
    from spark_h3_b200 import _lib

    schedule = np.array([1, 1, 65, 65, *([1] * 65)], dtype=np.int32)
    assert _lib.load().sb_reblock_plan(schedule.ctypes.data, len(schedule), 65 * 64, None, 0) < 0
    assert "2 to 64 children" in _lib.load().sb_last_error().decode()


def test_spark_reblock_rejects_unimplemented_options():
    import torch

    x = torch.zeros(1, 128, 128, dtype=torch.bfloat16)
    with pytest.raises(NotImplementedError, match="distance"):
        reblock.spark_reblock(x, grid_shape=(1, 1, 128), distance="euclidean")
    with pytest.raises(NotImplementedError, match="update_rule"):
        reblock.spark_reblock(x, grid_shape=(1, 1, 128), update_rule="medoid")
    with pytest.raises(TypeError):
        reblock.spark_reblock(x, grid_shape=(1, 1, 128), colour="blue")


@pytest.mark.parametrize("kwargs,match", [({"proxy_iterations": 3}, "proxy_iterations"),
                                          ({"seed_rule": "random"}, "seed_rule"),
                                          ({"update_rule": "median"}, "update_rule")])
def test_proxy_controls_reject_undefined_semantics(kwargs, match):
    """The reference's own cases (tests/test_reblock_proxy_controls.py:113-126), same messages."""
    import torch

    with pytest.raises(ValueError, match=match):
        reblock.spark_reblock(torch.zeros(1, 128, 128, dtype=torch.bfloat16), grid_shape=(1, 2, 64), **kwargs)


@pytest.mark.parametrize("excluded,match", [([[1]], "shape"), ([[1, 1]], "unique"), ([[1, 130]], "range")])
def test_frozen_excluded_indices_are_strictly_validated(excluded, match):
    """The reference's own cases (tests/test_reblock_proxy_controls.py:159-173), same messages."""
    import torch

    with pytest.raises(ValueError, match=match):
        reblock.validate_excluded(torch.tensor(excluded), 1, 130, torch.device("cpu"))
    ids = reblock.validate_excluded(torch.tensor([[77, 3]]), 1, 130, torch.device("cpu"))
    assert ids.dtype == torch.int32 and ids.tolist() == [[77, 3]]


def test_plan_proxy_controls():
    from spark_h3_b200 import _lib

    lib = _lib.load()
    h = build_reblock_hierarchy(4096, 16)
    schedule = reblock._schedule(h)
    n = lib.sb_reblock_plan(schedule.ctypes.data, len(schedule), 4096, None, 0)
    plan = np.zeros(n, dtype=np.int32)
    assert lib.sb_reblock_plan(schedule.ctypes.data, len(schedule), 4096, plan.ctypes.data, n) == n
    assert list(plan[6:8]) == [2, 0]  # the production controls
    for iterations, endpoint in ((0, 1), (1, 0), (4, 1), (2, 0)):
        assert lib.sb_reblock_plan_proxy(plan.ctypes.data, iterations, endpoint) == 0
        assert list(plan[6:8]) == [iterations, endpoint]
    for iterations, endpoint in ((3, 0), (-1, 0), (8, 0), (2, 2)):
        assert lib.sb_reblock_plan_proxy(plan.ctypes.data, iterations, endpoint) < 0
        assert list(plan[6:8]) == [2, 0]
    assert lib.sb_reblock_plan_proxy(plan.ctypes.data, 3, 0) < 0
    assert "proxy_iterations must be 0, 1, 2, or 4" in lib.sb_last_error().decode()


def test_reblock_reuse_across_layers(monkeypatch):
    """Groups of `spark_reblock_reuse_layers` layers share the first layer's permutations
    within one evaluation (spark_integration.py:941-988); a new evaluation rebuilds."""
    from spark_h3_b200 import attention
    from spark_h3_b200.config import H3SparseAttentionConfig
    from spark_h3_b200.processor import _Controller

    builds = []

    def fake_builder(q, k, video, grid, **kwargs):
        builds.append(q)
        return (f"qp{len(builds)}", f"qi{len(builds)}", f"kp{len(builds)}", None, f"h{len(builds)}")

    monkeypatch.setattr(attention._reblock, "qk_block_permutations", fake_builder)
    controller = _Controller(H3SparseAttentionConfig.spark(num_inference_steps=4, mode="full",
                                                           sol_route_topk_ratio=0.1))

    class Layout:
        grid = (1, 8, 8)

    def run(layer):
        return attention._reblock_permutations(controller, object(), object(), Layout, layer, 64)[0]

    controller.evaluation_index = 0
    assert [run(layer) for layer in range(4)] == ["qp1", "qp2", "qp3", "qp4"]  # default: no reuse
    controller.spark_reblock_reuse_layers = 2
    controller.spark_reblock_reuse_start_layer = 1
    assert [run(layer) for layer in range(6)] == ["qp5", "qp6", "qp6", "qp7", "qp7", "qp8"]
    assert controller.counts["sol_landmark_reuse_calls"] == 2
    controller.evaluation_index = 1
    assert run(1) == "qp9" and run(2) == "qp9"
    controller.reset()
    assert controller.spark_reblock_reuse_layers == 2  # settings survive reset, as in the reference


def test_public_spark_names_match_reference_exports():
    """h3_sparse_attention/__init__.py:12-36 and spark.py:34-39: spark_reblock, spark_reweight
    and spark_block (the initial public name of spark_reblock) from the package root and from
    the spark module, as the same objects."""
    import spark_h3_b200
    from spark_h3_b200 import spark

    assert spark_h3_b200.spark_block is spark_h3_b200.spark_reblock is reblock.spark_reblock
    assert spark.spark_reblock is spark_h3_b200.spark_reblock
    assert spark.spark_block is spark_h3_b200.spark_reblock
    assert spark.spark_reweight is spark_h3_b200.spark_reweight
    assert spark.install_h3_spark_attn is spark_h3_b200.install_h3_spark_attn
    for name in ("spark_reblock", "spark_reweight", "spark_block", "install_fp8", "Fp8Linear",
                 "convert_linear_to_fp8", "install_h3_spark_attn", "install_h3_sol_attn",
                 "install_h3_sparse_attention", "H3SparseAttentionConfig", "H3SparseAttentionPlugin"):
        assert name in spark_h3_b200.__all__, name


def test_tree_entry_points_name_themselves_in_errors():
    """Argument errors of the shared tree code name the entry point the caller used (no GPU:
    both are refused before any launch)."""
    from spark_h3_b200 import _lib

    lib = _lib.load()
    plan = np.zeros(16, dtype=np.int32)
    assert lib.sb_reblock_tree(None, 1, 128, 128, None, plan.ctypes.data, None, None, 0, None, None, None) < 0
    assert lib.sb_last_error().decode().startswith("sb_reblock_tree: null pointer")
    assert lib.sb_reblock_tree_frozen(None, 1, 128, 128, None, None, plan.ctypes.data, None, None, 0, None, None,
                                      None) < 0
    assert lib.sb_last_error().decode().startswith("sb_reblock_tree_frozen: null pointer")
    assert lib.sb_reblock_tree_frozen(None, 1, 130, 128, None, None, plan.ctypes.data, None, None, 0, None, None,
                                      None) < 0
    assert "excluded ids are required" in lib.sb_last_error().decode()


def _no_gpu() -> bool:
    import torch

    return not torch.cuda.is_available()


@pytest.mark.skipif(not _no_gpu(), reason="passes placeholder addresses; runs only where no GPU exists")
def test_remainder_entry_point_validates_its_arguments():
    """sb_reblock_remainder refuses bad arguments before any launch.  The non-null pointers are
    placeholders the checks reject before any use, so this runs only on a host without a GPU,
    where nothing could be launched on them."""
    from spark_h3_b200 import _lib

    lib = _lib.load()
    assert lib.sb_reblock_remainder(None, 1, 130, 128, None, 0, None, None) < 0
    assert "null pointer" in lib.sb_last_error().decode()
    fake = 1 << 20  # a non-null, aligned address that is never dereferenced: checks fail first
    assert lib.sb_reblock_remainder(fake, 1, 130, 64, fake, 8 * 130, fake, None) < 0
    assert "feature dimension must be 128" in lib.sb_last_error().decode()
    assert lib.sb_reblock_remainder(fake, 1, 130, 128, fake, 8 * 130 - 1, fake, None) < 0
    assert "workspace holds" in lib.sb_last_error().decode()
    assert lib.sb_reblock_remainder(fake, 1, 130, 128, fake, 8 * 130, None, None) < 0
    assert "null excluded buffer" in lib.sb_last_error().decode()
    assert lib.sb_reblock_remainder(fake, 1, 128, 128, fake, 8 * 128, None, None) == 0  # no remainder: nothing to do


def test_m2_side_is_validated():
    import torch

    with pytest.raises(ValueError, match="m2_side"):
        reblock._required_m2_side("diag", "independent")
    assert reblock._required_m2_side("query", "q_from_k") == "none"
    assert reblock._required_m2_side("both", "k_from_q") == "query"
    with pytest.raises(RuntimeError):  # CUDA tensors only
        reblock.remainder_ids(torch.zeros(1, 130, 128, dtype=torch.bfloat16))
