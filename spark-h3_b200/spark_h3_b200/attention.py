"""Spark sparse attention on packed BTHD tensors: the seam the C ABI replaces.

`spark_attention_bthd` has the contract of
h3_sparse_attention/spark_integration.py:883-1283 (video tokens first, context after; rows
past the last complete video block attend densely; output in packed order) and runs the
whole layer on the GPU through libsparkh3b200.so:
    pool Q -> global anchor -> pool K + summaries -> scores + Top-K -> sparse attention.
"""
from __future__ import annotations

import math

import torch

from . import ops
from . import reblock as _reblock
from .hierarchy import build_reblock_hierarchy, virtual_query_layout

BACKEND_TENSOR = "b200_sm100_fused_virtual_query"
BACKEND_SIMT = "b200_simt_virtual_query"


sparse_query_tokens = ops.sparse_query_tokens  # spark_integration.py:72-91


def reweight_flags(components: str) -> tuple[bool, bool]:
    """(anchor-weighted K/V, log-mass bias) for sol_reweight_components
    (sol_numerator_virtual_q.py:224-231)."""
    return components in ("full", "weights_only"), components in ("full", "bias_only")


def topk_density(stats: dict) -> dict:
    """Analytic density of a fixed Top-K budget (spark_integration.py:228-242)."""
    selected = min(stats["target_topk_blocks_per_query"], stats["candidate_video_blocks"])
    return dict(additional_topk_density=selected / stats["candidate_video_blocks"],
                effective_video_density=selected / stats["candidate_video_blocks"],
                effective_packed_density=(selected + stats["sink_blocks"]) / stats["blocks"])


def _check_inputs(q, k, v):
    if q.shape != k.shape or q.shape != v.shape:
        raise RuntimeError("Spark attention requires matching BTHD Q/K/V tensors")
    if not (q.is_contiguous() and k.is_contiguous() and v.is_contiguous()):
        raise RuntimeError("Spark attention requires contiguous BTHD Q/K/V tensors")
    if q.device.type != "cuda":
        raise RuntimeError("Spark-H3 requires CUDA tensors")
    if q.dtype not in (torch.bfloat16, torch.float32) or q.shape[-1] not in (64, 128) or k.dtype != q.dtype:
        raise RuntimeError("the B200 Spark kernels take BF16 or FP32 Q/K/V with head dimension 64 or 128; "
                           f"got dtype={q.dtype}, head_dim={q.shape[-1]}")
    capability = tuple(torch.cuda.get_device_capability(q.device))
    if capability != (10, 0):
        raise RuntimeError(f"the B200 Spark kernels are built for SM100 only; got SM{capability[0]}{capability[1]}")


def spark_attention_bthd(controller, q_bthd, k_bthd, v_bthd, layout, layer, *, return_bthd: bool = True,
                         workspace: torch.Tensor | None = None):
    cfg = controller.config
    _check_inputs(q_bthd, k_bthd, v_bthd)
    if cfg.sol_route_topk_ratio is None:
        raise RuntimeError("the B200 path implements Top-K routed Spark attention; set sol_route_topk_ratio")
    if cfg.sol_tail_granularity == "block8x8" and cfg.sol_reweight_summary_math != "tensorcore":
        raise ValueError("block8x8 currently supports tensorcore numeric mode only")
    B, T, H, D = q_bthd.shape
    head_budgets = _head_budgets(getattr(controller, "head_topk_budget", None), H, q_bthd.device)
    block = cfg.sol_block_size
    video = int(layout.video_tokens)
    if video < block:
        raise RuntimeError(f"Spark routing requires at least one complete {block}-token video block")
    tail_mode = "legacy_full" if cfg.sol_legacy_full_query else cfg.sol_video_tail_mode
    query_tokens = sparse_query_tokens(T, video, block, tail_mode)
    query_blocks = query_tokens // block
    candidates = video // block
    nb = math.ceil(T / block)
    sink_tokens = layout.sequence_length - video
    sink_first = video // block
    sink_last = math.ceil((video + sink_tokens) / block) if sink_tokens else sink_first
    topk = ops.target_topk(cfg.sol_route_topk_ratio, candidates)
    if head_budgets is not None and (sink_tokens or video % block):
        # head_budget.py:16-18: with per-head budgets the partial video block and all
        # conditioning stay exact.
        sink_first, sink_last = candidates, nb
    weighted_kv, mass_bias = reweight_flags(cfg.sol_reweight_components)
    anchor_dtype = torch.float32 if cfg.sol_global_anchor_dtype == "float32" or q_bthd.dtype == torch.float32 \
        else q_bthd.dtype

    query_inverse = None
    if cfg.sol_landmark_preprocess:
        _check_reblock(cfg, q_bthd, block)
        q_perm, query_inverse, k_perm, hierarchy = _reblock_permutations(controller, q_bthd, k_bthd, layout,
                                                                          layer, video)
        controller.landmark_reblock_hierarchy = hierarchy
        q_bthd = ops.headwise_permute(q_bthd, q_perm, video)
        k_bthd = ops.headwise_permute(k_bthd, k_perm, video)
        v_bthd = ops.headwise_permute(v_bthd, k_perm, video)
        controller.counts["sol_landmark_preprocess_calls"] += 1

    # Padding fills after any reblock permutation (spark_integration.py:1173-1187); the anchor
    # covers the complete video blocks only (landmark_virtual_q.py:30-41).
    # With sol_legacy_full_query the partial final block keeps the mean of its real rows, video
    # and context alike (spark_integration.py:925-933; _sol_topk_policy_scores pools every token).
    qc = ops.pool_queries(q_bthd, block)
    if tail_mode == "pad":
        qc = ops.padded_query_means(q_bthd, qc, video, query_tokens, block)
    anchor = ops.query_anchor(qc, block, candidates, anchor_dtype)
    kc, ak, av, lm = ops.pool_keys_summaries(k_bthd, v_bthd, anchor, block, weighted_kv=weighted_kv,
                                             mass_bias=mass_bias, summary_math=cfg.sol_reweight_summary_math,
                                             logmass_key=cfg.sol_reweight_logmass_key)
    packed, _ = ops.route_topk(qc, kc, query_blocks, candidates, topk, workspace=workspace, want_indices=False,
                               head_budgets=head_budgets)
    out = ops.pooled_tail_attention(q_bthd, k_bthd, v_bthd, block, packed, ak, av, lm, anchor,
                                    query_tokens=query_tokens, sink_first=sink_first, sink_last=sink_last,
                                    local_radius=cfg.kernel_local_radius, tail_granularity=cfg.sol_tail_granularity,
                                    weighted_kv=weighted_kv, mass_bias=mass_bias,
                                    logmass_key=cfg.sol_reweight_logmass_key)
    # Rows past dense_start attend densely (spark_integration.py:1238-1260): the kernel covers
    # rows past the sparse prefix; the context rows that padded it are recomputed here.
    dense_start = video if query_tokens > video else query_tokens
    if query_tokens > video:
        ops.dense_rows_attention(q_bthd, k_bthd, v_bthd, video, query_tokens, out)

    controller.sol_backend = BACKEND_TENSOR if (q_bthd.dtype == torch.bfloat16 and D == 128) else BACKEND_SIMT
    controller.counts["sol_topk_packed_route_calls"] += 1
    controller.counts["sol_virtual_query_calls"] += 1
    if not cfg.sol_landmark_preprocess:
        controller.counts["sol_identity_virtual_query_calls"] += 1
        if cfg.sol_spark_mode == "reweight_only":
            controller.counts["sol_identity_reweight_calls"] += 1
    controller.counts["sol_topk_calls"] += 1
    if T > dense_start:
        controller.counts["sol_dense_context_queries"] += 1
    if cfg.sol_landmark_preprocess:
        key = ("reblock_global_anchor", T, video, controller.landmark_reblock_hierarchy)
        topology = controller._virtual_query_layout_cache.get(key)
        if topology is None:
            topology = dict(virtual_query_layout(video, T, 99, hierarchy=controller.landmark_reblock_hierarchy)
                            ["metadata"])
            controller._virtual_query_layout_cache[key] = topology
        controller.sol_virtual_query_layout = topology
        controller.counts["sol_virtual_query_fused_permute_calls"] += 1
        key = None
    else:
        key = ("identity_global_anchor", T, video, layout.grid)
    topology = controller._virtual_query_layout_cache.get(key) if key is not None else None
    if key is not None and topology is None and video >= 64:
        hierarchy = build_reblock_hierarchy(video, cfg.landmark_tree_v2_children, grid_shape=tuple(layout.grid),
                                            fanout_mode=cfg.landmark_tree_v2_fanout_mode)
        topology = dict(virtual_query_layout(video, T, 99, hierarchy=hierarchy)["metadata"])
        controller._virtual_query_layout_cache[key] = topology
    if key is not None and topology is not None:
        controller.sol_virtual_query_layout = {**topology, "layout": "identity_physical_order",
                                               "anchor_policy": "global"}
    if cfg.sol_log_density and controller.sol_route_density is None:
        mode = "per_head_exact_topk" if head_budgets is not None else "gemm_exact_topk_packed_external"
        stats = dict(block_size=block, blocks=nb, candidate_video_blocks=candidates, query_video_blocks=query_blocks,
                     sink_blocks=max(0, nb - candidates), route_threshold_mode=mode,
                     route_topk_ratio=cfg.sol_route_topk_ratio, target_topk_blocks_per_query=topk,
                     packed_route_words=math.ceil(nb / 32))
        stats.update(topk_density(stats))
        controller.sol_route_density = stats
    if query_inverse is not None:
        out = ops.headwise_permute(out, query_inverse, video)
    return out if return_bthd else out.permute(0, 2, 1, 3).contiguous()


def _head_budgets(budget, heads: int, device: torch.device) -> torch.Tensor | None:
    """The controller's per-head Top-K budgets (processor.py:787-796 sets them from a
    head_budget_allocator) as int32 [H] on the layer's device; one budget per head is
    required, as in head_budget.py:9-10."""
    if budget is None:
        return None
    budget = torch.as_tensor(budget)
    if tuple(budget.shape) != (heads,):
        raise ValueError("expected one budget per head")
    return budget.to(device=device, dtype=torch.int32).contiguous()


_REBLOCK_DEFAULTS = dict(
    landmark_tree_v2_distance="cosine", landmark_tree_v2_order_mode="parent_order", landmark_tree_v2_mean_mode="raw",
    landmark_tree_v2_moment_mode="raw", landmark_tree_v2_group_size=1, landmark_tree_v2_landmark_mode="midpoint",
    landmark_tree_v2_landmark_count=32, landmark_tree_v2_aggregation="linear",
    landmark_tree_v2_m2_estimator="hilbert_midpoint", landmark_tree_v2_proxy_update_rule="mean")


def _reblock_permutations(controller, q_bthd, k_bthd, layout, layer: int, video: int):
    """Query/key permutations of one layer, shared by groups of layers when the controller
    asks for it (spark_integration.py:941-988): with `spark_reblock_reuse_layers` = R > 1,
    layers from `spark_reblock_reuse_start_layer` on form groups of R, and every layer of a
    group after its first reuses the first layer's permutations within the same evaluation."""
    cfg = controller.config
    reuse_layers = int(getattr(controller, "spark_reblock_reuse_layers", 1))
    reuse_start = int(getattr(controller, "spark_reblock_reuse_start_layer", 0))
    group = (layer - reuse_start) // reuse_layers if reuse_layers > 1 and layer >= reuse_start else None
    key = (controller.evaluation_index, group)
    cached = getattr(controller, "spark_last_reblock", None)
    group_start = reuse_start + group * reuse_layers if group is not None else layer
    if group is not None and layer != group_start and cached is not None and cached[0] == key:
        controller.counts["sol_landmark_reuse_calls"] += 1
        return cached[1]
    q_perm, query_inverse, k_perm, _, hierarchy = _reblock.qk_block_permutations(
        q_bthd, k_bthd, video, layout.grid, children=cfg.landmark_tree_v2_children,
        fanout_mode=cfg.landmark_tree_v2_fanout_mode, final_fanout=cfg.landmark_tree_v2_final_fanout,
        root_fanout=cfg.landmark_tree_v2_root_fanout, ridge=cfg.rope_sol_key_ridge_epsilon,
        initial_order=cfg.landmark_tree_v2_initial_order, proxy_iterations=cfg.landmark_tree_v2_proxy_iterations,
        seed_rule=cfg.landmark_tree_v2_proxy_seed_rule, layout_reuse=cfg.landmark_tree_v2_layout_reuse,
        m2_side=cfg.landmark_tree_v2_m2_side)
    controller.counts["rope_sol_landmark_tree_v2_key_assignments"] += 1
    controller.counts["rope_sol_landmark_tree_v2_query_assignments"] += 1
    result = (q_perm, query_inverse, k_perm, hierarchy)
    if group is not None:
        controller.spark_last_reblock = (key, result)
    return result


def _check_reblock(cfg, q, block: int) -> None:
    """The B200 reblock implements the production landmark-tree-v2 configuration."""
    if block != 64:
        raise NotImplementedError("landmark reblocking builds 64-token blocks; use sol_block_size=64")
    if q.dtype != torch.bfloat16 or q.shape[-1] != 128:
        raise RuntimeError("the B200 reblock path takes bf16 Q/K/V with head dimension 128")
    for name, default in _REBLOCK_DEFAULTS.items():
        value = getattr(cfg, name)
        if value != default:
            raise NotImplementedError(f"the B200 reblock path implements {name}={default!r}; got {value!r}")


def spark_reweight(a: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, block: int = 64,
                   summary_math: str = "tensorcore", logmass_key: str = "stored",
                   reweight_components: str = "full"):
    """Anchor-conditioned summaries for query representatives a[B, P, H, D] and keys/values
    k, v[B, T, H, D]: returns (AK, AV [B, P, H, NB, D], LM [B, P, H, NB]) like the reference's
    spark_reweight = virtual_summaries (sol_numerator_virtual_q.py:334-353)."""
    if a.ndim != 4 or k.ndim != 4 or v.shape != k.shape or a.shape[0] != k.shape[0] or a.shape[2:] != k.shape[2:]:
        raise ValueError("requires nonempty A[BP H D] and matching K/V[BT H D]")
    weighted_kv, mass_bias = reweight_flags(reweight_components)
    parts = []
    for p in range(a.shape[1]):
        _, ak, av, lm = ops.pool_keys_summaries(k, v, a[:, p].contiguous(), block, weighted_kv=weighted_kv,
                                                mass_bias=mass_bias, want_kc=False, summary_math=summary_math,
                                                logmass_key=logmass_key)
        parts.append((ak, av, lm))
    return tuple(torch.stack([part[i] for part in parts], dim=1) for i in range(3))
