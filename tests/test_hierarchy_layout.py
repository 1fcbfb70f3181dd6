"""Reblock hierarchy planning and the packed layout against the reference's outputs
(tests/golden/*.json) and its known-answer cases."""
import hashlib
import json
from pathlib import Path

import pytest
import torch

from spark_h3_b200.hierarchy import build_reblock_hierarchy, power_of_two_child_budgets, virtual_query_layout
from spark_h3_b200.layout import packed_layout

GOLDEN = Path(__file__).resolve().parent / "golden"


def test_hierarchy_matches_reference_plans():
    for case in json.loads((GOLDEN / "hierarchy.json").read_text()):
        children = tuple(case["children"]) if isinstance(case["children"], list) else case["children"]
        h = build_reblock_hierarchy(case["video_tokens"], children, fanout_mode=case["fanout_mode"],
                                    final_fanout=case["final_fanout"])
        levels = [list(map(list, level)) for level in h.levels]
        assert hashlib.sha256(json.dumps(levels).encode()).hexdigest() == case["levels_digest"]
        if case["levels"] is not None:
            assert levels == case["levels"]
        assert [[[size, list(b)] for size, b in rnd] for rnd in h.split_budgets] == case["split_budgets"]
        layout = virtual_query_layout(case["video_tokens"], case["video_tokens"] + 999, 99, hierarchy=h)
        assert [list(r) for r in layout["ranges"]] == case["layout_ranges"]
        for key, value in case["layout_metadata"].items():
            assert layout["metadata"][key] == value


def test_global_frontier_of_the_default_spark_hierarchy():
    h = build_reblock_hierarchy(72576, 16, grid_shape=(72, 24, 42))
    layout = virtual_query_layout(72576, 73565, 99, hierarchy=h)
    assert h.roots == ((0, 1134),)
    assert layout["metadata"]["active_size_counts"] == {72576: 1}
    assert layout["metadata"]["global_video_representative"]
    # Halving the capacities, larger half first: 1134 -> 567+567 -> 284+283+284+283 -> ...
    assert power_of_two_child_budgets(1134, (16,)) == (71,) * 7 + (70,) + (71,) * 7 + (70,)


def test_layout_matches_reference_cases():
    for case in json.loads((GOLDEN / "layout.json").read_text()):
        tags = torch.tensor(case["tags"])
        pos = torch.tensor(case["positions"])
        kwargs = {}
        if case["kind"] == "indexed":
            kwargs = dict(video_indices=torch.tensor(case["video_indices"]),
                          timestep_indices=torch.tensor(case["timestep_indices"]),
                          text_indices=torch.tensor(case["text_indices"]), sparse_video_scope=case["scope"])
        lay = packed_layout(tags, pos, **kwargs)
        assert lay.permutation.tolist() == case["permutation"]
        assert list(lay.grid) == case["grid"]
        assert lay.video_tokens == case["video_tokens"]
        assert torch.equal(lay.permutation[lay.inverse_permutation], torch.arange(len(case["tags"])))


def test_target_suffix_and_heterogeneous_condition_planes():
    tags = torch.tensor([0, 0, 1, 2, 0, 0])
    positions = torch.tensor([[0, 0, 0], [0, 0, 1], [0, 0, 0], [0, 0, 0], [0, 0, 0], [0, 0, 1]])
    lay = packed_layout(tags, positions, video_indices=torch.tensor([0, 1, 4, 5]),
                        timestep_indices=torch.zeros(6, dtype=torch.long), text_indices=torch.tensor([2]))
    assert lay.video_tokens == 2 and lay.permutation.tolist() == [4, 5, 0, 1, 2, 3]
    # condition: two time planes with different grids; target: one 2x2 plane
    tags = torch.tensor([0, 0, 0, 0, 0, 0, 1, 0, 0, 0, 0])
    positions = torch.tensor([[0, 0, 0], [0, 0, 1], [1, 0, 0], [1, 0, 1], [1, 1, 0], [1, 1, 1], [0, 0, 0],
                              [2, 0, 0], [2, 0, 1], [2, 1, 0], [2, 1, 1]])
    lay = packed_layout(tags, positions, video_indices=torch.tensor([0, 1, 2, 3, 4, 5, 7, 8, 9, 10]),
                        timestep_indices=torch.tensor([0, 0, 0, 0, 0, 0, 1, 1, 1, 1, 1]),
                        text_indices=torch.tensor([6]), sparse_video_scope="target_and_condition")
    assert lay.grid == (1, 1, 10) and lay.video_tokens == 10
    assert lay.target_video_tokens == 4 and lay.condition_video_tokens == 6
    assert lay.permutation.tolist() == [0, 1, 2, 3, 4, 5, 7, 8, 9, 10, 6]


def test_layout_rejects_malformed_inputs():
    with pytest.raises(ValueError, match="unexpected shapes"):
        packed_layout(torch.zeros(4, dtype=torch.long), torch.zeros(3, 3, dtype=torch.long))
    with pytest.raises(ValueError, match="no video tokens"):
        packed_layout(torch.ones(4, dtype=torch.long), torch.zeros(4, 3, dtype=torch.long))
    with pytest.raises(ValueError, match="dense grid"):
        packed_layout(torch.zeros(3, dtype=torch.long), torch.tensor([[0, 0, 0], [0, 1, 1], [0, 0, 1]]))
