"""Configuration of the Spark / Sol sparse attention plugin.

Field names, defaults, the `spark()` / `sol()` presets and the validation messages follow
h3_sparse_attention/processor.py:17-535 so that code (and tests) written against the
reference's `H3SparseAttentionConfig` work unchanged.  One field is new:
`sol_block_size` (64, the reference's fixed block, or 128).
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Literal

from . import hierarchy as _h


def resolve_denoise_steps(num_inference_steps, num_denoise_steps, *, default):
    """Actual denoising evaluations from either count (processor.py:17-37)."""
    if num_inference_steps is not None and num_denoise_steps is not None:
        raise ValueError("set either num_denoise_steps or num_inference_steps, not both")
    if num_denoise_steps is not None:
        if type(num_denoise_steps) is not int or num_denoise_steps < 1:
            raise ValueError("num_denoise_steps must be a positive integer")
        return num_denoise_steps
    if num_inference_steps is None:
        return default
    if type(num_inference_steps) is not int or num_inference_steps < 2:
        raise ValueError("num_inference_steps must be an integer of at least 2")
    return num_inference_steps - 1


def _require(cond, message, exc=ValueError):
    if not cond:
        raise exc(message)


def _choice(value, options, message):
    _require(value in options, message)


@dataclass(frozen=True)
class H3SparseAttentionConfig:
    method: str = "sol"
    total_evaluations: int = 19
    warmup_mode: Literal["warmup_ratio", "warmup_steps"] = "warmup_ratio"
    warmup_ratio: float = 0.2
    warmup_steps: int = 4
    warmup_percent: float | None = None
    sol_tau: float = 1.0
    sol_thresh_type: str = "diag"
    sol_kv_splits: int = 1
    sol_dense_layers: int = 1
    sol_min_tokens: int = 0
    sol_extra_dense_evaluations: tuple = ()
    sol_extra_dense_layers: tuple = ()
    sol_force_local_blocks: bool | None = None
    sol_exact_block_radius: int | None = None
    sol_tail_granularity: str = "query"
    sol_global_anchor_dtype: str = "float32"
    sol_reweight_summary_math: str = "tensorcore"
    sol_reweight_logmass_key: str = "stored"
    sol_reweight_components: str = "full"
    sol_spark_mode: str | None = None
    sol_route_topk_ratio: float | None = None
    sol_route_topk_cutoff_mode: str = "gemm_radix"
    sol_route_topk_execution: str = "packed_external_no_route_qk"
    sol_sparse_video_scope: str = "target"
    sol_video_tail_mode: str = "dense"
    sol_legacy_full_query: bool = False
    sol_log_density: bool = True
    sol_landmark_preprocess: bool = False
    sol_landmark_preprocess_version: str = "v1"
    sol_virtual_query_levels_up: int | None = None
    sol_virtual_query_target_blocks: int | None = None
    sol_virtual_query_min_blocks: int = 4
    sol_virtual_query_max_blocks: int = 12
    sol_virtual_query_fused_permute: bool = True
    sol_virtual_query_route_score: str = "native_mean"
    landmark_tree_v2_initial_order: str = "flat"
    landmark_tree_v2_distance: str = "cosine"
    landmark_tree_v2_order_mode: str = "parent_order"
    landmark_tree_v2_mean_mode: str = "raw"
    landmark_tree_v2_moment_mode: str = "raw"
    landmark_tree_v2_group_size: object = 1
    landmark_tree_v2_children: object = None
    landmark_tree_v2_fanout: object = None
    landmark_tree_v2_final_fanout: object = None
    landmark_tree_v2_root_fanout: int | None = None
    landmark_tree_v2_landmark_mode: str = "midpoint"
    landmark_tree_v2_landmark_count: int = 32
    landmark_tree_v2_midpoint_direction_mode: str = "legacy"
    landmark_tree_v2_aggregation: str = "linear"
    rope_sol_key_ridge_epsilon: float = 1e-3
    landmark_tree_v2_m2_side: str = "both"
    landmark_tree_v2_m2_estimator: str = "hilbert_midpoint"
    landmark_tree_v2_proxy_iterations: int = 2
    landmark_tree_v2_proxy_seed_rule: str = "farthest_pair"
    landmark_tree_v2_proxy_update_rule: str = "mean"
    landmark_tree_v2_layout_reuse: str = "independent"
    sol_route_global_weighted_mean: bool = False
    sol_route_global_weighted_side: str = "both"
    landmark_tree_v2_fanout_mode: str = "power_of_two_fanout"
    sol_block_size: int = 64

    def __post_init__(self):
        self._check_schedule()
        self._check_dense_policy()
        self._check_sparse_policy()
        self._check_virtual_query()
        self._check_landmark_tree()

    # --------------------------------------------------------------- validation
    def _set(self, name, value):
        object.__setattr__(self, name, value)

    def _check_schedule(self):
        _require(self.method == "sol", "this package supports method='sol' only")
        _require(type(self.total_evaluations) is int and self.total_evaluations >= 1,
                 "total_evaluations must be a positive integer")
        _choice(self.warmup_mode, ("warmup_ratio", "warmup_steps"),
                "warmup_mode must be 'warmup_ratio' or 'warmup_steps'")
        _require(math.isfinite(self.warmup_ratio) and 0 <= self.warmup_ratio <= 1,
                 "warmup_ratio must be finite and lie in [0, 1]")
        _require(type(self.warmup_steps) is int and self.warmup_steps >= 0,
                 "warmup_steps must be a nonnegative integer")
        if self.warmup_percent is not None:
            _require(math.isfinite(self.warmup_percent) and 0 <= self.warmup_percent <= 100,
                     "warmup_percent must be finite and lie in [0, 100]")
            _require(self.warmup_mode == "warmup_ratio" and self.warmup_ratio == 0.2 and self.warmup_steps == 4,
                     "warmup_percent cannot be combined with warmup_mode, warmup_ratio, or warmup_steps")
            self._set("warmup_ratio", self.warmup_percent / 100)

    def _check_dense_policy(self):
        _require(math.isfinite(self.sol_tau) and self.sol_tau >= 0, "sol_tau must be finite and nonnegative")
        _choice(self.sol_thresh_type, ("diag", "exact"), "sol_thresh_type must be 'diag' or 'exact'")
        _require(type(self.sol_kv_splits) is int and self.sol_kv_splits >= 1, "sol_kv_splits must be a positive integer")
        _require(type(self.sol_dense_layers) is int and self.sol_dense_layers >= 0,
                 "sol_dense_layers must be a nonnegative integer")
        _require(type(self.sol_min_tokens) is int and self.sol_min_tokens >= 0,
                 "sol_min_tokens must be a nonnegative integer")
        evals = self.sol_extra_dense_evaluations
        _require(type(evals) is tuple and all(type(e) is int and 0 <= e < self.total_evaluations for e in evals),
                 "sol_extra_dense_evaluations must be a tuple of evaluation indices in [0, total_evaluations)")
        self._set("sol_extra_dense_evaluations", tuple(sorted(set(evals))))
        layers = self.sol_extra_dense_layers
        _require(type(layers) is tuple and all(type(x) is int and x >= 0 for x in layers),
                 "sol_extra_dense_layers must be a tuple of nonnegative layer indices")
        self._set("sol_extra_dense_layers", tuple(sorted(set(layers))))
        _require(self.sol_force_local_blocks is None or type(self.sol_force_local_blocks) is bool,
                 "sol_force_local_blocks must be bool")
        radius = self.sol_exact_block_radius
        _require(radius is None or (type(radius) is int and radius >= 0),
                 "sol_exact_block_radius must be None or a nonnegative integer")
        _require(radius is None or self.sol_force_local_blocks is None,
                 "set sol_exact_block_radius or sol_force_local_blocks, not both")
        _require(radius is None or self.sol_route_topk_ratio is not None, "sol_exact_block_radius requires Top-K routing")
        _require(self.sol_block_size in (64, 128), "sol_block_size must be 64 or 128")

    def _check_sparse_policy(self):
        _choice(self.sol_tail_granularity, ("query", "block", "block8x8"),
                "sol_tail_granularity must be 'query', 'block', or 'block8x8'")
        _choice(self.sol_global_anchor_dtype, ("bfloat16", "float32"),
                "sol_global_anchor_dtype must be 'bfloat16' or 'float32'")
        _choice(self.sol_reweight_summary_math, ("tensorcore", "comfy_fp32"), "invalid sol_reweight_summary_math")
        _choice(self.sol_reweight_logmass_key, ("stored", "pre_round"), "invalid sol_reweight_logmass_key")
        _choice(self.sol_reweight_components, ("full", "weights_only", "bias_only", "none"),
                "invalid sol_reweight_components")
        _choice(self.sol_spark_mode, (None, "topk_only", "reblock_only", "reweight_only", "full"),
                "sol_spark_mode must be topk_only, reblock_only, reweight_only, full, or None")
        ratio = self.sol_route_topk_ratio
        _require(ratio is None or 0 < ratio <= 1, "sol_route_topk_ratio must lie in (0, 1]")
        _choice(self.sol_route_topk_cutoff_mode, ("gemm_radix", "gaussian_moments"),
                "invalid sol_route_topk_cutoff_mode")
        execution = self.sol_route_topk_execution
        if execution == "packed_external":
            raise ValueError("sol_route_topk_execution='packed_external' was removed because it is bitwise-equivalent "
                             "but slower; use 'packed_external_no_route_qk'")
        if execution in ("threshold", "fused"):
            raise ValueError(f"sol_route_topk_execution={execution!r} is disabled; use 'packed_external_no_route_qk' "
                             "so exact Top-K selections are encoded and consumed as packed routes")
        _require(execution == "packed_external_no_route_qk", "invalid sol_route_topk_execution")
        _choice(self.sol_sparse_video_scope, ("target", "target_and_condition"),
                "sol_sparse_video_scope must be 'target' or 'target_and_condition'")
        _choice(self.sol_video_tail_mode, ("dense", "pad"), "sol_video_tail_mode must be 'dense' or 'pad'")
        _require(type(self.sol_legacy_full_query) is bool, "sol_legacy_full_query must be bool", TypeError)
        _require(not (self.sol_legacy_full_query and self.sol_video_tail_mode != "dense"),
                 "sol_legacy_full_query is incompatible with sol_video_tail_mode='pad'")
        _require(not self.sol_landmark_preprocess or self.sol_landmark_preprocess_version == "v2",
                 "this port supports landmark preprocessing version 'v2' only")
        self._set("landmark_tree_v2_fanout_mode", _h.normalize_fanout_mode(self.landmark_tree_v2_fanout_mode))
        _require(type(self.sol_route_global_weighted_mean) is bool, "sol_route_global_weighted_mean must be bool",
                 TypeError)
        _choice(self.sol_route_global_weighted_side, ("both", "query", "key"),
                "sol_route_global_weighted_side must be both, query, or key")
        _require(not self.sol_route_global_weighted_mean or ratio is not None,
                 "global weighted routing requires Top-K routing")
        _require(math.isfinite(self.rope_sol_key_ridge_epsilon) and self.rope_sol_key_ridge_epsilon >= 0,
                 "rope_sol_key_ridge_epsilon must be finite and nonnegative")

    def _check_virtual_query(self):
        _choice(self.landmark_tree_v2_m2_side, ("both", "query", "key", "none"),
                "landmark_tree_v2_m2_side must be both, query, key, or none")
        _choice(self.landmark_tree_v2_m2_estimator, ("hilbert_midpoint", "flat64_block_mean", "flat64_midpoint_1",
                                                     "flat64_midpoint_2", "flat64_midpoint_4", "flat64_mean_diag",
                                                     "full"), "invalid landmark_tree_v2_m2_estimator")
        _choice(self.landmark_tree_v2_proxy_iterations, (0, 1, 2, 4),
                "landmark_tree_v2_proxy_iterations must be 0, 1, 2, or 4")
        _choice(self.landmark_tree_v2_proxy_seed_rule, ("farthest_pair", "endpoint_order"),
                "invalid landmark_tree_v2_proxy_seed_rule")
        _choice(self.landmark_tree_v2_proxy_update_rule, ("mean", "medoid"), "invalid landmark_tree_v2_proxy_update_rule")
        _choice(self.landmark_tree_v2_layout_reuse, ("independent", "q_from_k", "k_from_q"),
                "invalid landmark_tree_v2_layout_reuse")
        _require(not (self.sol_exact_block_radius is not None and self.sol_landmark_preprocess
                      and self.landmark_tree_v2_layout_reuse == "independent"),
                 "sol_exact_block_radius with reblock requires landmark_tree_v2_layout_reuse='q_from_k' or 'k_from_q'")
        _choice(self.sol_virtual_query_route_score, ("native_mean", "mean", "weighted_k", "weighted_mass"),
                "invalid sol_virtual_query_route_score")
        virtual = self.sol_virtual_query_levels_up is not None or self.sol_virtual_query_target_blocks is not None
        if self.sol_spark_mode is not None:
            reblock = self.sol_spark_mode in ("reblock_only", "full")
            reweight = self.sol_spark_mode in ("reweight_only", "full")
            _require(self.sol_route_topk_ratio is not None, "Spark component modes require Top-K routing")
            _require(self.sol_landmark_preprocess == reblock,
                     f"sol_spark_mode={self.sol_spark_mode!r} requires sol_landmark_preprocess={reblock}")
            _require((self.sol_reweight_components != "none") == reweight,
                     f"sol_spark_mode={self.sol_spark_mode!r} has an incompatible sol_reweight_components value")
            _require(self.sol_virtual_query_target_blocks is None and self.sol_virtual_query_levels_up == 99
                     and self.sol_virtual_query_route_score == "native_mean",
                     "public Spark modes use one global anchor; target-block, multi-level, and reweighted-route "
                     "topologies are disabled")
        numeric_default = (self.sol_reweight_summary_math == "tensorcore" and self.sol_reweight_logmass_key == "stored"
                           and self.sol_reweight_components == "full")
        _require(numeric_default or virtual, "reweight numeric ablations require virtual query summaries")
        _require(self.sol_tail_granularity == "query" or virtual, "block tail requires virtual query summaries")
        _require(self.sol_virtual_query_route_score == "native_mean" or virtual,
                 "reweighted routing requires virtual query summaries")
        _require(self.sol_virtual_query_levels_up is None or self.sol_virtual_query_target_blocks is None,
                 "choose either sol_virtual_query_levels_up or sol_virtual_query_target_blocks")
        if self.sol_virtual_query_levels_up is not None:
            _require(type(self.sol_virtual_query_levels_up) is int and self.sol_virtual_query_levels_up >= 0,
                     "sol_virtual_query_levels_up must be None or a nonnegative integer")
        if self.sol_virtual_query_target_blocks is not None:
            _require(type(self.sol_virtual_query_target_blocks) is int,
                     "sol_virtual_query_target_blocks must be an integer or None")
            _require(type(self.sol_virtual_query_min_blocks) is int and type(self.sol_virtual_query_max_blocks) is int
                     and 1 <= self.sol_virtual_query_min_blocks <= self.sol_virtual_query_target_blocks
                     <= self.sol_virtual_query_max_blocks, "virtual query blocks require 1 <= min <= target <= max")
        if virtual:
            _require(self.sol_spark_mode is not None
                     or (self.sol_landmark_preprocess and self.sol_landmark_preprocess_version == "v2"),
                     "virtual query summaries require LMv2 Sol preprocessing")
            _require(self.sol_route_topk_ratio is not None or self.sol_virtual_query_route_score == "native_mean",
                     "tau routing with virtual query summaries requires native_mean scores")
        _require(not (self.sol_video_tail_mode == "pad" and self.sol_route_topk_ratio is None and not virtual),
                 "sol_video_tail_mode='pad' requires Top-K or virtual-query routing")

    def _check_landmark_tree(self):
        _choice(self.landmark_tree_v2_moment_mode, ("raw", "unit"), "landmark_tree_v2_moment_mode must be raw or unit")
        _choice(self.landmark_tree_v2_mean_mode, ("raw", "input_unit", "metric_unit"),
                "landmark_tree_v2_mean_mode must be raw, input_unit or metric_unit")
        _require(self.landmark_tree_v2_mean_mode == "raw" or self.landmark_tree_v2_distance == "cosine",
                 "input-unit means require cosine distance")
        _h.normalize_initial_order(self.landmark_tree_v2_initial_order)
        if self.landmark_tree_v2_fanout is not None:
            if self.landmark_tree_v2_children is not None and (
                    _h.normalize_fanout(self.landmark_tree_v2_children, None)
                    != _h.normalize_fanout(self.landmark_tree_v2_fanout, None)):
                raise ValueError("use landmark_tree_v2_fanout or landmark_tree_v2_children, not conflicting values")
            children = self.landmark_tree_v2_fanout
        elif self.landmark_tree_v2_children is None:
            children = 16
        else:
            children = self.landmark_tree_v2_children
        self._set("landmark_tree_v2_children", _h.normalize_fanout(children, None))
        if self.landmark_tree_v2_fanout is not None:
            self._set("landmark_tree_v2_fanout", self.landmark_tree_v2_children)
        if self.landmark_tree_v2_root_fanout is not None:
            _h.resolve_root_fanout(self.landmark_tree_v2_children, self.landmark_tree_v2_root_fanout)
        if self.landmark_tree_v2_final_fanout is not None:
            self._set("landmark_tree_v2_final_fanout", _h.normalize_final_fanout(self.landmark_tree_v2_final_fanout))
        _choice(self.landmark_tree_v2_landmark_count, (32, 64, 128, 256),
                "landmark_tree_v2_landmark_count must be 32, 64, 128, or 256")
        _choice(self.landmark_tree_v2_landmark_mode, ("mean", "midpoint"),
                "landmark_tree_v2_landmark_mode must be mean or midpoint")
        if self.landmark_tree_v2_midpoint_direction_mode == "fused":
            raise ValueError("landmark_tree_v2_midpoint_direction_mode='fused' is disabled; Spark experiments are "
                             "fixed to 'legacy'")
        _require(self.landmark_tree_v2_midpoint_direction_mode == "legacy",
                 "landmark_tree_v2_midpoint_direction_mode must be legacy")
        _require(self.landmark_tree_v2_aggregation in ("linear", "max")
                 and not (self.landmark_tree_v2_aggregation == "max" and self.landmark_tree_v2_distance != "cosine"),
                 "max aggregation requires cosine distance")
        _choice(self.landmark_tree_v2_distance, ("euclidean", "cosine"),
                "landmark_tree_v2_distance must be euclidean or cosine")
        self._set("landmark_tree_v2_order_mode", _h.normalize_order_mode(self.landmark_tree_v2_order_mode))
        self._set("landmark_tree_v2_group_size", _h.normalize_group_size(self.landmark_tree_v2_group_size))
        _require(self.sol_virtual_query_route_score == "native_mean" or self.sol_local_blocks_enabled,
                 "reweighted route scores require sol_force_local_blocks=True")

    # --------------------------------------------------------------- derived
    @property
    def sol_local_blocks_enabled(self):
        if self.sol_exact_block_radius is not None:
            return True
        if self.sol_force_local_blocks is not None:
            return self.sol_force_local_blocks
        return not self.sol_landmark_preprocess

    @property
    def sol_local_block_radius(self):
        """-1 disables local retention; a nonnegative value is the symmetric radius."""
        if self.sol_exact_block_radius is not None:
            return self.sol_exact_block_radius
        return 1 if self.sol_local_blocks_enabled else -1

    @property
    def sol_local_block_policy(self):
        if self.sol_exact_block_radius is not None:
            return self.sol_exact_block_radius
        return self.sol_local_blocks_enabled

    @property
    def kernel_local_radius(self):
        """Radius the sparse kernel applies to packed external routes: an explicit
        sol_exact_block_radius only (a boolean policy is ignored for external routes,
        sol_attn/sm90/mainloop.py:115-122)."""
        return self.sol_exact_block_radius if self.sol_exact_block_radius is not None else -1

    @property
    def dense_evaluations(self):
        if self.warmup_mode == "warmup_steps":
            return min(self.total_evaluations, self.warmup_steps)
        return min(self.total_evaluations, math.ceil(self.total_evaluations * self.warmup_ratio))

    # --------------------------------------------------------------- presets
    @staticmethod
    def _validate_warmup_overrides(overrides):
        if "warmup_percent" in overrides and any(n in overrides for n in ("warmup_mode", "warmup_ratio",
                                                                           "warmup_steps")):
            raise ValueError("warmup_percent cannot be combined with warmup_mode, warmup_ratio, or warmup_steps")

    @classmethod
    def sol(cls, num_inference_steps=None, *, num_denoise_steps=None, **overrides):
        cls._validate_warmup_overrides(overrides)
        total = resolve_denoise_steps(num_inference_steps, num_denoise_steps, default=19)
        return cls(total_evaluations=total, **overrides)

    @classmethod
    def spark(cls, num_inference_steps=None, *, num_denoise_steps=None, mode="full", **overrides):
        """One of the four fixed-layout/reblock x global-reweight modes (processor.py:422-512)."""
        cls._validate_warmup_overrides(overrides)
        if mode not in ("topk_only", "reblock_only", "reweight_only", "full"):
            raise ValueError("mode must be topk_only, reblock_only, reweight_only, or full")
        if "sol_spark_mode" in overrides:
            raise ValueError("pass mode= instead of sol_spark_mode")
        retired = sorted({"sol_virtual_query_target_blocks", "sol_virtual_query_min_blocks",
                          "sol_virtual_query_max_blocks", "sol_virtual_query_levels_up",
                          "sol_virtual_query_route_score", "sol_landmark_preprocess"}.intersection(overrides))
        if retired:
            raise ValueError("public Spark modes fix global-anchor topology and reblocking; remove legacy overrides: "
                             + ", ".join(retired))
        reblock = mode in ("reblock_only", "full")
        reweight = mode in ("reweight_only", "full")
        if "sol_reweight_components" in overrides and (overrides["sol_reweight_components"] != "none") != reweight:
            raise ValueError("sol_reweight_components conflicts with the selected Spark mode")
        defaults = dict(
            sol_dense_layers=0, sol_route_topk_ratio=0.1, sol_route_topk_cutoff_mode="gemm_radix",
            sol_route_topk_execution="packed_external_no_route_qk", sol_min_tokens=8192,
            sol_global_anchor_dtype="bfloat16", sol_spark_mode=mode,
            sol_reweight_components="full" if reweight else "none", sol_landmark_preprocess=reblock,
            sol_landmark_preprocess_version="v2", landmark_tree_v2_children=16,
            landmark_tree_v2_midpoint_direction_mode="legacy", sol_virtual_query_target_blocks=None,
            sol_virtual_query_levels_up=99, sol_virtual_query_route_score="native_mean")
        if overrides.get("landmark_tree_v2_fanout") is not None and "landmark_tree_v2_children" not in overrides:
            defaults.pop("landmark_tree_v2_children")
        defaults.update(overrides)
        total = resolve_denoise_steps(num_inference_steps, num_denoise_steps, default=19)
        return cls(total_evaluations=total, **defaults)
