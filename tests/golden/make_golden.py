"""Generate the golden fixtures in this directory from the reference's own code.

Run in a container that has a read-only checkout of the reference, with its path in
$SPARK_H3_REFERENCE; the tests only read the committed fixtures and never import the
reference.  Inputs are regenerated deterministically by the tests from the recorded seeds
(torch CPU generator) and checked against the recorded SHA-256 digests first.

    SPARK_H3_REFERENCE=<reference checkout> python tests/golden/make_golden.py

Fixtures:
  hierarchy.json  build_reblock_hierarchy / virtual_query_layout (reblock_hierarchy.py,
                  landmark_virtual_q.py) for a set of fanout schedules
  layout.json     _packed_layout (processor.py:550-688) on tag/position patterns
  route_*.npz     _sol_topk_policy_scores + _sol_topk_route_from_scores
                  (spark_integration.py:94-175): the selected block sets per row, and the
                  gap between the k-th and (k+1)-th score of every row
  route_config1_b64.npz  the same reference route at production size (
                  grid (31, 48, 84), N = 124,992, H = 32, D = 128, bf16, 64-token blocks,
                  k = 195 of 1953): per row a 64-bit digest (the first 8 bytes of the SHA-256
                  of the ascending int32 block indices) and the k-th/(k+1)-th score gap, plus
                  the full sets of 256 seeded sample rows
  head_budget.npz route_with_head_budgets (head_budget.py:7-19): per-head budgets on seeded
                  scores quantised to force ties at the cut ("ties"), and on the fp32
                  scores of _sol_topk_policy_scores for synthetic Q/K with a context suffix
                  ("pipeline"); the boolean routes over every key block
  summaries.npz   the Triton _summaries kernel (sol_numerator_virtual_q.py:93-135) run under
                  TRITON_INTERPRET=1 in fp32 at D=128
  attention.npz   the explicit exact/summary softmax of tests/test_spark_installer.py:559-570
                  applied to the reference's route and summaries (fp32)
  reblock_tree.npz  recursive_landmark_tree_v2_reference (landmark_tree_v2.py:790-832) on
                  seeded bf16 features: the permutation per case
  reblock_tree_modes.npz  the same on the other two fanout modes, arbitrary_fanout and
                  power_of_two_arbitrary_final (reblock_hierarchy.py:124-160), whose nodes
                  split into non-power-of-two child counts over landmark_v2_terminal.py's
                  split topology; the permutation and the hierarchy's split budgets per case
  reblock_tree_proxy.npz  the same with the proxy controls of landmark_v2_terminal.py:43-50
                  (proxy_iterations 0 / 1 / 4, seed_rule endpoint_order), which the reference
                  always runs through node_split_reference
  reblock_tree_frozen.npz  the same with a caller-chosen protected remainder (excluded_indices,
                  landmark_tree_clustering.py:99-119): the seeded ids and the permutation
  reblock_m2.npz  the paired Q/K reblock with the M2 ablations (landmark_tree_v2_m2_side none /
                  key / query, spark_integration.py:450-693: raw features on the sides without
                  the factor, the baseline tail frozen) and a shared layout, on clustered Q/K
  reblock_qk.npz  the full paired Q/K reblock (_landmark_tree_v2_qk_block_permutations,
                  spark_integration.py:735-851, CPU controller, mode "full") on clustered
                  synthetic Q/K: Hilbert metric samples, the Cholesky factors, the bf16
                  features the tree consumed and the Q/K permutations
"""
from __future__ import annotations

import hashlib
import json
import math
import os
import sys
from pathlib import Path

os.environ.setdefault("TRITON_INTERPRET", "1")
HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
if not os.environ.get("SPARK_H3_REFERENCE"):
    raise SystemExit("set SPARK_H3_REFERENCE to the reference checkout")
REFERENCE = Path(os.environ["SPARK_H3_REFERENCE"])
sys.path[:0] = [str(REFERENCE), str(ROOT), str(ROOT / "spark-h3_b200")]

import numpy as np  # noqa: E402
import torch  # noqa: E402


def digest(t: torch.Tensor) -> str:
    t = t.detach().cpu().contiguous()
    raw = t.view(torch.int16).numpy() if t.dtype == torch.bfloat16 else t.numpy()
    return hashlib.sha256(raw.tobytes()).hexdigest()


def hierarchy_cases():
    from h3_sparse_attention.landmark_virtual_q import virtual_query_layout
    from h3_sparse_attention.reblock_hierarchy import build_reblock_hierarchy

    cases = []
    for video, children, mode, final in [
        (72576, 16, "power_of_two_fanout", None), (4096, 16, "power_of_two_fanout", None),
        (245952, 16, "power_of_two_fanout", None), (124992, 16, "power_of_two_fanout", None),
        (124992, (8, 4), "power_of_two_fanout", None), (245952, 8, "arbitrary_fanout", None),
        (245952, 16, "arbitrary_fanout", 12), (100000, 4, "power_of_two_arbitrary_final", 6),
        (64 * 37, 2, "power_of_two_fanout", None), (64 * 1000, 32, "arbitrary_fanout", None),
    ]:
        h = build_reblock_hierarchy(video, children, fanout_mode=mode, final_fanout=final)
        layout = virtual_query_layout(video, video + 999, 99, hierarchy=h)
        levels = [list(map(list, level)) for level in h.levels]
        cases.append(dict(video_tokens=video, children=children, fanout_mode=mode, final_fanout=final,
                          levels=levels if video <= 8192 else None,
                          levels_digest=hashlib.sha256(json.dumps(levels).encode()).hexdigest(),
                          split_budgets=[[[size, list(b)] for size, b in rnd] for rnd in h.split_budgets],
                          layout_ranges=[list(r) for r in layout["ranges"]],
                          layout_metadata={k: layout["metadata"][k] for k in (
                              "active_virtual_blocks", "total_virtual_blocks", "global_video_representative",
                              "total_split_levels")}))
    return cases


def layout_cases():
    from h3_sparse_attention.processor import _packed_layout

    out = []
    # video grid (3, 4, 5) shuffled, 7 text tokens interleaved
    g = torch.Generator().manual_seed(5)
    grid = torch.cartesian_prod(torch.arange(3), torch.arange(4), torch.arange(5))
    order = torch.randperm(60, generator=g)
    tags = torch.cat([torch.zeros(60, dtype=torch.long), torch.ones(7, dtype=torch.long)])
    pos = torch.cat([grid[order], torch.zeros(7, 3, dtype=torch.long)])
    mix = torch.randperm(67, generator=g)
    tags, pos = tags[mix], pos[mix]
    lay = _packed_layout(tags, pos)
    out.append(dict(kind="tags_only", tags=tags.tolist(), positions=pos.tolist(),
                    permutation=lay.permutation.tolist(), grid=list(lay.grid), video_tokens=lay.video_tokens))
    # structural target suffix with conditioning video
    tags = torch.tensor([0, 0, 1, 2, 0, 0, 0, 0])
    pos = torch.tensor([[0, 0, 0], [0, 0, 1], [0, 0, 0], [0, 0, 0], [0, 1, 1], [0, 0, 0], [0, 1, 0], [0, 0, 1]])
    for scope in ("target", "target_and_condition"):
        ts = torch.tensor([1, 1, 0, 0, 0, 0, 0, 0]) if scope == "target_and_condition" else torch.zeros(8).long()
        kwargs = dict(video_indices=torch.tensor([0, 1, 4, 5, 6, 7]), timestep_indices=ts,
                      text_indices=torch.tensor([2]), sparse_video_scope=scope)
        lay = _packed_layout(tags, pos, **kwargs)
        out.append(dict(kind="indexed", scope=scope, tags=tags.tolist(), positions=pos.tolist(),
                        video_indices=[0, 1, 4, 5, 6, 7], timestep_indices=ts.tolist(), text_indices=[2],
                        permutation=lay.permutation.tolist(), grid=list(lay.grid), video_tokens=lay.video_tokens,
                        target_video_tokens=lay.target_video_tokens,
                        condition_video_tokens=lay.condition_video_tokens))
    return out


def block_mean(x: torch.Tensor, block: int) -> torch.Tensor:
    """fp32 block mean (the reference's query centroid; for keys it is then rounded)."""
    B, T, H, D = x.shape
    nb = math.ceil(T / block)
    pad = torch.nn.functional.pad(x.float(), (0, 0, 0, 0, 0, nb * block - T))
    counts = torch.full((nb,), float(block))
    counts[-1] = T - (nb - 1) * block
    return pad.view(B, nb, block, H, D).sum(2) / counts.view(1, nb, 1, 1)


def route_case(name, grid, heads, dim, dtype, q_scale, seed):
    from h3_sparse_attention.spark_integration import _sol_topk_policy_scores, _sol_topk_route_from_scores
    from spark_h3_b200.synthetic import make_qkv

    q, k, v = make_qkv(grid, heads, dim, seed=seed, dtype=dtype, q_scale=q_scale)
    T = q.shape[1]
    kc = block_mean(k, 64).to(dtype)
    scores, adjacent, cand, qblocks, target = _sol_topk_policy_scores(q, kc, video_tokens=T, topk_ratio=0.1)
    route = _sol_topk_route_from_scores(scores, adjacent, candidate_blocks=cand, target_topk=target,
                                        video_tokens=T, sink_tokens=0)
    s = scores[..., :cand]
    top = torch.sort(s, dim=-1, descending=True).values
    gap = (top[..., target - 1] - top[..., target]).float() if target < cand else torch.full(top.shape[:-1], np.inf)
    np.savez_compressed(HERE / f"route_{name}.npz", route=route[:, :qblocks, :, :cand].numpy().astype(np.uint8),
                        gap=gap.numpy().astype(np.float32), kc_digest=np.array(digest(kc)),
                        q_digest=np.array(digest(q)), k_digest=np.array(digest(k)), target=np.array(target),
                        meta=np.array(json.dumps(dict(grid=grid, heads=heads, dim=dim, dtype=str(dtype),
                                                      q_scale=q_scale, seed=seed))))


def row_digests(indices: np.ndarray) -> np.ndarray:
    """uint64 per row: the first 8 bytes (little endian) of the SHA-256 of the row's ascending
    int32 indices."""
    rows = np.ascontiguousarray(np.sort(indices.reshape(-1, indices.shape[-1]), axis=-1).astype("<i4"))
    return np.array([int.from_bytes(hashlib.sha256(r.tobytes()).digest()[:8], "little") for r in rows],
                    dtype=np.uint64)


def route_config1_case():
    """The reference's fp32 route at BASELINE config 1 with 64-token blocks (its only block
    size): Q/K from the seeded generator the tests share, key centroids as the fp32 block mean
    rounded to bf16 (the _reduce_kc_kernel rule, sol_attn/preprocess.py:16-52)."""
    from h3_sparse_attention.spark_integration import _sol_topk_policy_scores, _sol_topk_route_from_scores
    from spark_h3_b200.synthetic import make_qkv

    grid, heads, dim, seed = (31, 48, 84), 32, 128, 0
    q, k = make_qkv(grid, heads, dim, seed=seed, dtype=torch.bfloat16, q_scale=dim ** -0.5, with_v=False)
    T = q.shape[1]
    kc = block_mean(k, 64).to(torch.bfloat16)
    scores, adjacent, cand, qblocks, target = _sol_topk_policy_scores(q, kc, video_tokens=T, topk_ratio=0.1)
    route = _sol_topk_route_from_scores(scores, adjacent, candidate_blocks=cand, target_topk=target,
                                        video_tokens=T, sink_tokens=0)
    sel = route[0, :qblocks, :, :cand]                       # [QB, H, C]
    assert int(sel.sum(-1).min()) == target and int(sel.sum(-1).max()) == target
    idx = torch.nonzero(sel.reshape(-1, cand))[:, 1].reshape(-1, target).numpy()  # ascending per row
    s = scores[0, :qblocks, :, :cand]
    top = torch.topk(s, target + 1, dim=-1).values
    gap = (top[..., target - 1] - top[..., target]).reshape(-1).numpy().astype(np.float32)
    rng = np.random.default_rng(1)
    sample = np.sort(rng.choice(idx.shape[0], 256, replace=False)).astype(np.int32)
    np.savez_compressed(HERE / "route_config1_b64.npz", row_digest=row_digests(idx), gap=gap,
                        sample_rows=sample, sample_sets=idx[sample].astype(np.int16),
                        q_digest=np.array(digest(q)), k_digest=np.array(digest(k)), target=np.array(target),
                        meta=np.array(json.dumps(dict(grid=grid, heads=heads, dim=dim, dtype="torch.bfloat16",
                                                      q_scale=dim ** -0.5, seed=seed, block=64,
                                                      topk_ratio=0.1))))


def head_budget_fixture():
    from h3_sparse_attention.head_budget import route_with_head_budgets
    from h3_sparse_attention.spark_integration import _sol_topk_policy_scores
    from spark_h3_b200.synthetic import make_qkv

    out = {}
    # ties: scores on a grid of 8 values, so every cut falls inside a group of equal scores;
    # budgets include 0 and one above the candidate count.
    gen = torch.Generator().manual_seed(23)
    scores = torch.randint(0, 8, (1, 12, 5, 44), generator=gen).float() / 4.0
    budgets = torch.tensor([0, 1, 7, 40, 50])
    route = route_with_head_budgets(scores, budgets, 40, 40 * 64 + 17, 0)  # partial video block
    out.update(ties_scores=scores.numpy(), ties_budgets=budgets.numpy().astype(np.int32),
               ties_route=route.numpy().astype(np.uint8), ties_candidates=np.array(40),
               ties_video=np.array(40 * 64 + 17))
    # pipeline: fp32 policy scores of synthetic Q/K; 100 context tokens follow the video.
    grid, heads, dim = (2, 16, 40), 4, 128
    q, k, _ = make_qkv(grid, heads, dim, seed=29, dtype=torch.bfloat16, q_scale=dim ** -0.5)
    T = q.shape[1]
    video = T - 100
    kc = block_mean(k, 64).to(torch.bfloat16)
    scores, _, cand, qblocks, target = _sol_topk_policy_scores(q, kc, video_tokens=video, topk_ratio=0.1)
    budgets = torch.tensor([3, 0, 12, 21])
    route = route_with_head_budgets(scores, budgets, cand, video, T - video)
    out.update(pipe_route=route[:, :qblocks].numpy().astype(np.uint8), pipe_budgets=budgets.numpy().astype(np.int32),
               pipe_video=np.array(video), pipe_candidates=np.array(cand), pipe_q_digest=np.array(digest(q)),
               pipe_k_digest=np.array(digest(k)),
               pipe_meta=np.array(json.dumps(dict(grid=grid, heads=heads, dim=dim, seed=29, q_scale=dim ** -0.5))))
    np.savez_compressed(HERE / "head_budget.npz", **out)


def summaries_and_attention():
    import triton
    from h3_sparse_attention.sol_numerator_virtual_q import _summaries
    from h3_sparse_attention.spark_integration import _sol_topk_policy_scores, _sol_topk_route_from_scores

    gen = torch.Generator().manual_seed(17)
    B, T, H, D = 1, 1000, 2, 128
    q = torch.randn(B, T, H, D, generator=gen) * D ** -0.5
    k = torch.randn(B, T, H, D, generator=gen)
    v = torch.randn(B, T, H, D, generator=gen)
    a = q[:, :960].mean(1, keepdim=True)  # anchor over the complete 64-token blocks
    n = triton.cdiv(T, 64)
    ak = torch.empty(B, 1, H, n, D)
    av = torch.empty_like(ak)
    lm = torch.empty(B, 1, H, n)
    _summaries[(1, n, B * H)](a, k, v, ak, av, lm, T, H, n, 1, a.stride(0), a.stride(1), 0, 1, 16, H, 0, True, False,
                              True, True, False, num_warps=4)
    np.savez_compressed(HERE / "summaries.npz", a=a.numpy(), ak=ak.numpy(), av=av.numpy(), lm=lm.numpy(),
                        q_digest=np.array(digest(q)), k_digest=np.array(digest(k)), v_digest=np.array(digest(v)))
    kc = block_mean(k, 64)
    scores, adjacent, cand, qblocks, target = _sol_topk_policy_scores(q, kc, video_tokens=960, topk_ratio=0.2)
    route = _sol_topk_route_from_scores(scores, adjacent, candidate_blocks=cand, target_topk=target,
                                        video_tokens=960, sink_tokens=40)
    out = torch.empty_like(q)
    for h in range(H):
        for blk in range(960 // 64):
            rows = slice(blk * 64, (blk + 1) * 64)
            exact = route[0, blk, h].repeat_interleave(64)[:T]
            approx = ~route[0, blk, h]
            keys = torch.cat([k[0, exact, h], ak[0, 0, h, approx]])
            vals = torch.cat([v[0, exact, h], av[0, 0, h, approx]])
            logits = q[0, rows, h] @ keys.T / D ** 0.5
            logits[:, int(exact.sum()):] += lm[0, 0, h, approx]
            out[0, rows, h] = logits.softmax(-1) @ vals
        out[0, 960:, h] = torch.softmax(q[0, 960:, h] @ k[0, :, h].T / D ** 0.5, -1) @ v[0, :, h]
    rows = np.r_[0:128, 896:1000]  # two routed blocks, the last routed block and the dense tail
    np.savez_compressed(HERE / "attention.npz", route=route[0].numpy().astype(np.uint8), rows=rows,
                        out=out[0, rows].numpy(), target=np.array(target))


REBLOCK_TREE_CASES = [
    # (name, tokens, dim, children, grid, initial order, seed)
    ("remainder", 4133, 128, 16, (1, 1, 4133), "flat", 0),
    ("grid8k", 8192, 128, 16, (2, 64, 64), "flat", 1),
    ("hilbert4", 3000, 64, 4, (3, 20, 50), "hilbert_thw", 2),
    ("tiny", 130, 128, 16, (1, 2, 65), "flat", 3),
    ("two_rounds", 20000, 128, 16, (5, 40, 100), "flat", 4),
    ("fanout8", 6016, 128, 8, (4, 32, 47), "tile_t4h4w4", 5),
]


def reblock_tree_fixture():
    from h3_sparse_attention.landmark_tree_v2 import recursive_landmark_tree_v2_reference

    out = {}
    for name, tokens, dim, children, grid, order, seed in REBLOCK_TREE_CASES:
        g = torch.Generator().manual_seed(seed)
        x = torch.randn(2, tokens, dim, generator=g).to(torch.bfloat16)
        ref = recursive_landmark_tree_v2_reference(x, grid_shape=grid, max_children=children, initial_order=order)
        out[f"{name}_perm"] = ref.permutation.numpy().astype(np.int32)
        out[f"{name}_digest"] = np.array(digest(x))
    np.savez_compressed(HERE / "reblock_tree.npz", **out)


REBLOCK_TREE_MODE_CASES = [
    # (name, tokens, children, final fanout, fanout mode, grid, initial order, seed)
    ("arb_two_rounds", 20000, 16, None, "arbitrary_fanout", (5, 40, 100), "flat", 21),
    ("arb_fanout8", 6016, 8, None, "arbitrary_fanout", (4, 32, 47), "tile_t4h4w4", 22),
    ("p2final_8_16", 6016, 8, 16, "power_of_two_arbitrary_final", (4, 32, 47), "flat", 23),
    ("arb_final12", 13000, 16, 12, "arbitrary_fanout", (1, 1, 13000), "flat", 24),
    ("arb_root3", 12352, 4, 3, "arbitrary_fanout", (2, 32, 193), "hilbert_thw", 25),
    ("arb_fanout64", 12800, 64, None, "arbitrary_fanout", (2, 80, 80), "flat", 26),
    ("arb_final24", 20160, 32, 24, "arbitrary_fanout", (5, 63, 64), "flat", 27),
]


def reblock_tree_modes_fixture():
    from h3_sparse_attention.landmark_tree_v2 import recursive_landmark_tree_v2_reference

    out = {}
    for name, tokens, children, final_fanout, mode, grid, order, seed in REBLOCK_TREE_MODE_CASES:
        g = torch.Generator().manual_seed(seed)
        x = torch.randn(2, tokens, 128, generator=g).to(torch.bfloat16)
        ref = recursive_landmark_tree_v2_reference(x, grid_shape=grid, max_children=children,
                                                   final_fanout=final_fanout, fanout_mode=mode,
                                                   initial_order=order)
        out[f"{name}_perm"] = ref.permutation.numpy().astype(np.int32)
        out[f"{name}_digest"] = np.array(digest(x))
        out[f"{name}_budgets"] = np.array(json.dumps([[list(map(int, b)) for _, b in rnd]
                                                      for rnd in ref.hierarchy.split_budgets]))
    np.savez_compressed(HERE / "reblock_tree_modes.npz", **out)


REBLOCK_TREE_PROXY_CASES = [
    # (name, tokens, children, fanout mode, grid, proxy_iterations, seed_rule, seed)
    ("iter0_endpoint", 4096, 4, "power_of_two_fanout", (1, 64, 64), 0, "endpoint_order", 31),
    ("iter1_farthest", 8192, 16, "power_of_two_fanout", (2, 64, 64), 1, "farthest_pair", 32),
    ("iter4_farthest", 6016, 8, "power_of_two_fanout", (4, 32, 47), 4, "farthest_pair", 33),
    ("iter1_endpoint", 4133, 16, "power_of_two_fanout", (1, 1, 4133), 1, "endpoint_order", 34),
    ("iter0_arbitrary", 6016, 8, "arbitrary_fanout", (4, 32, 47), 0, "farthest_pair", 35),
    ("iter4_endpoint_arbitrary", 20000, 16, "arbitrary_fanout", (5, 40, 100), 4, "endpoint_order", 36),
]


def reblock_tree_proxy_fixture():
    from h3_sparse_attention.landmark_tree_v2 import recursive_landmark_tree_v2_reference

    out = {}
    for name, tokens, children, mode, grid, iterations, seed_rule, seed in REBLOCK_TREE_PROXY_CASES:
        g = torch.Generator().manual_seed(seed)
        x = torch.randn(2, tokens, 128, generator=g).to(torch.bfloat16)
        ref = recursive_landmark_tree_v2_reference(x, grid_shape=grid, max_children=children, fanout_mode=mode,
                                                   proxy_iterations=iterations, seed_rule=seed_rule)
        out[f"{name}_perm"] = ref.permutation.numpy().astype(np.int32)
        out[f"{name}_digest"] = np.array(digest(x))
    np.savez_compressed(HERE / "reblock_tree_proxy.npz", **out)


REBLOCK_TREE_FROZEN_CASES = [
    # (name, tokens, children, grid, initial order, seed)
    ("frozen_remainder", 4133, 16, (1, 1, 4133), "flat", 41),
    ("frozen_two", 130, 16, (1, 2, 65), "flat", 42),
    ("frozen_hilbert", 20000, 16, (5, 40, 100), "hilbert_thw", 43),
]


def reblock_tree_frozen_fixture():
    from h3_sparse_attention.landmark_tree_v2 import recursive_landmark_tree_v2_reference

    out = {}
    for name, tokens, children, grid, order, seed in REBLOCK_TREE_FROZEN_CASES:
        g = torch.Generator().manual_seed(seed)
        x = torch.randn(2, tokens, 128, generator=g).to(torch.bfloat16)
        excluded = torch.stack([torch.randperm(tokens, generator=g)[:tokens % 64] for _ in range(2)])
        ref = recursive_landmark_tree_v2_reference(x, grid_shape=grid, max_children=children, initial_order=order,
                                                   excluded_indices=excluded)
        out[f"{name}_perm"] = ref.permutation.numpy().astype(np.int32)
        out[f"{name}_excluded"] = excluded.numpy().astype(np.int32)
        out[f"{name}_digest"] = np.array(digest(x))
    np.savez_compressed(HERE / "reblock_tree_frozen.npz", **out)


def reblock_qk_fixture():
    from types import SimpleNamespace

    from h3_sparse_attention.landmark_direction import landmark_direction_factors
    from h3_sparse_attention.mahalanobis_kmeans import hilbert_midpoint_sample_indices
    from h3_sparse_attention.processor import H3SparseAttentionConfig, _Controller
    from h3_sparse_attention.spark_integration import _landmark_tree_v2_qk_block_permutations
    from spark_h3_b200.synthetic import make_qkv

    grid, heads, dim = (2, 16, 40), 1, 128
    q, k, _ = make_qkv(grid, heads, dim, seed=7, dtype=torch.bfloat16, clustered=True)
    T = q.shape[1]
    cfg = H3SparseAttentionConfig.spark(num_inference_steps=4, mode="full", sol_route_topk_ratio=0.1)
    controller = _Controller(cfg)
    layout = SimpleNamespace(video_tokens=T, grid=grid, sequence_length=T)
    qp, qi, kp, ki, _, _ = _landmark_tree_v2_qk_block_permutations(controller, q, k, layout)
    samples = hilbert_midpoint_sample_indices(grid, T // 64, device="cpu")
    flat_q = q.permute(0, 2, 1, 3).reshape(heads, T, dim)
    flat_k = k.permute(0, 2, 1, 3).reshape(heads, T, dim)
    lq, lk = landmark_direction_factors(flat_q, flat_k, samples, ridge=cfg.rope_sol_key_ridge_epsilon)
    features = torch.cat([torch.bmm(flat_k, lq.to(torch.bfloat16)), torch.bmm(flat_q, lk.to(torch.bfloat16))])
    np.savez_compressed(HERE / "reblock_qk.npz", grid=np.array(grid), heads=np.array(heads),
                        q_digest=np.array(digest(q)), k_digest=np.array(digest(k)),
                        samples=samples.numpy().astype(np.int32),
                        samples_big=hilbert_midpoint_sample_indices((61, 48, 84), 245952 // 64,
                                                                    device="cpu").numpy().astype(np.int32),
                        factors=torch.cat([lq, lk]).numpy(),
                        features=features.view(torch.int16).numpy().view(np.uint16),
                        q_perm=qp.numpy().astype(np.int32), k_perm=kp.numpy().astype(np.int32),
                        q_inv=qi.numpy().astype(np.int32), k_inv=ki.numpy().astype(np.int32))


REBLOCK_M2_CASES = [
    # (name, grid, heads, m2_side, layout_reuse, seed)
    ("none_even", (2, 16, 40), 2, "none", "independent", 7),
    ("none_rem", (2, 16, 41), 2, "none", "independent", 8),
    ("key_rem", (2, 16, 41), 2, "key", "independent", 9),
    ("query_rem", (2, 16, 41), 2, "query", "independent", 10),
    ("shared_none_rem", (2, 16, 41), 2, "none", "q_from_k", 11),
]


def reblock_m2_fixture():
    from types import SimpleNamespace

    from h3_sparse_attention.processor import H3SparseAttentionConfig, _Controller
    from h3_sparse_attention.spark_integration import _landmark_tree_v2_qk_block_permutations
    from spark_h3_b200.synthetic import make_qkv

    out = {}
    for name, grid, heads, m2_side, reuse, seed in REBLOCK_M2_CASES:
        q, k, _ = make_qkv(grid, heads, 128, seed=seed, dtype=torch.bfloat16, clustered=True)
        T = q.shape[1]
        cfg = H3SparseAttentionConfig.spark(num_inference_steps=4, mode="full", sol_route_topk_ratio=0.1,
                                            landmark_tree_v2_m2_side=m2_side, landmark_tree_v2_layout_reuse=reuse)
        layout = SimpleNamespace(video_tokens=T, grid=grid, sequence_length=T)
        qp, qi, kp, ki, _, _ = _landmark_tree_v2_qk_block_permutations(_Controller(cfg), q, k, layout)
        out[f"{name}_q_perm"] = qp.numpy().astype(np.int32)
        out[f"{name}_k_perm"] = kp.numpy().astype(np.int32)
        out[f"{name}_q_digest"] = np.array(digest(q))
        out[f"{name}_k_digest"] = np.array(digest(k))
    np.savez_compressed(HERE / "reblock_m2.npz", **out)


def main():
    (HERE / "hierarchy.json").write_text(json.dumps(hierarchy_cases()))
    (HERE / "layout.json").write_text(json.dumps(layout_cases()))
    route_case("config0", (4, 32, 32), 4, 64, torch.float32, 1.0, 0)
    route_case("bf16_d128", (2, 32, 64), 2, 128, torch.bfloat16, 128 ** -0.5, 1)
    route_config1_case()
    head_budget_fixture()
    summaries_and_attention()
    reblock_tree_fixture()
    reblock_tree_modes_fixture()
    reblock_tree_proxy_fixture()
    reblock_tree_frozen_fixture()
    reblock_m2_fixture()
    reblock_qk_fixture()
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    if len(sys.argv) > 1:
        for name in sys.argv[1:]:  # a subset, e.g. route_config1_case
            globals()[name]()
    else:
        main()
