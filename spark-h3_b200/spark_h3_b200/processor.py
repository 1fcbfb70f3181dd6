"""Reversible installation of the B200 Spark attention processor on a MiniMax-H3 transformer.

Mirrors h3_sparse_attention/processor.py:691-1144: the evaluation controller and its forward
pre-hook (packed layout per evaluation, warm-up accounting), the attention processor with
its dense gates, and the context-managed plugin with the same installer signatures.
"""
from __future__ import annotations

from collections import Counter
from typing import Any

import torch

from .attention import spark_attention_bthd
from .config import H3SparseAttentionConfig
from .layout import packed_layout


class _Controller:
    def __init__(self, config: H3SparseAttentionConfig):
        self.config = config
        # Reblock reuse across layers (spark_integration.py:944-945); kept over reset().
        self.spark_reblock_reuse_layers = 1
        self.spark_reblock_reuse_start_layer = 0
        self.reset()

    def reset(self):
        self.evaluation_index = -1
        self.layout = None
        self.counts = Counter()
        self.sol_backend = None
        self.rope_sol_key_clustering_static = {}
        self._virtual_query_layout_cache = {}
        self.landmark_reblock_hierarchy = None
        self.sol_virtual_query_layout = None
        self.sol_route_density = None
        self.exact_block_verbose_accumulator = None
        self.head_topk_budget = None
        self.spark_reblock_frozen_tail_indices = None
        self.spark_last_reblock = None

    def begin_forward(self, _module, args, kwargs):
        """Forward pre-hook: count the evaluation and rebuild the packed layout."""
        self.evaluation_index += 1
        if self.evaluation_index >= self.config.total_evaluations:
            raise RuntimeError("received more transformer evaluations than configured; "
                               "call plugin.reset() before another pipeline invocation")

        def argument(name, index):
            value = kwargs.get(name)
            return args[index] if value is None and len(args) > index else value

        tags = argument("token_tags", 5)
        positions = argument("position_ids", 6)
        if tags is None or positions is None:
            raise RuntimeError("H3 Sol-Attn requires token_tags/position_ids")
        self.layout = packed_layout(tags, positions, video_indices=argument("video_indices", 7),
                                    timestep_indices=argument("timestep_indices", 4),
                                    text_indices=argument("text_indices", 9),
                                    sparse_video_scope=self.config.sol_sparse_video_scope)

    @property
    def is_warmup(self):
        return self.evaluation_index < self.config.dense_evaluations

    def summary(self) -> dict[str, Any]:
        cfg = self.config
        layout = self.layout
        return dict(
            method="sol", sol_backend=self.sol_backend, completed_evaluations=self.evaluation_index + 1,
            total_evaluations=cfg.total_evaluations, warmup_mode=cfg.warmup_mode, warmup_ratio=cfg.warmup_ratio,
            warmup_steps=cfg.warmup_steps, min_tokens=cfg.sol_min_tokens, dense_evaluations=cfg.dense_evaluations,
            sol_extra_dense_evaluations=cfg.sol_extra_dense_evaluations,
            sol_extra_dense_layers=cfg.sol_extra_dense_layers, processor_calls=dict(self.counts),
            sol_route_density=self.sol_route_density, exact_block_verbose=None,
            sol_virtual_query_layout=self.sol_virtual_query_layout,
            sol_force_local_blocks=cfg.sol_local_blocks_enabled, sol_tail_granularity=cfg.sol_tail_granularity,
            sol_landmark_preprocess=cfg.sol_landmark_preprocess,
            landmark_tree_v2_children=cfg.landmark_tree_v2_children,
            landmark_tree_v2_fanout_mode=cfg.landmark_tree_v2_fanout_mode,
            landmark_tree_v2_midpoint_direction_mode=cfg.landmark_tree_v2_midpoint_direction_mode,
            sol_sparse_video_scope=cfg.sol_sparse_video_scope,
            sparse_video_tokens=None if layout is None else layout.video_tokens,
            target_video_tokens=None if layout is None else layout.target_video_tokens,
            condition_video_tokens=None if layout is None else layout.condition_video_tokens,
            landmark_tree_v2_m2_side=cfg.landmark_tree_v2_m2_side,
            landmark_tree_v2_m2_estimator=cfg.landmark_tree_v2_m2_estimator,
            landmark_tree_v2_proxy_iterations=cfg.landmark_tree_v2_proxy_iterations,
            landmark_tree_v2_proxy_seed_rule=cfg.landmark_tree_v2_proxy_seed_rule,
            landmark_tree_v2_proxy_update_rule=cfg.landmark_tree_v2_proxy_update_rule,
            landmark_tree_v2_layout_reuse=cfg.landmark_tree_v2_layout_reuse,
            sol_block_size=cfg.sol_block_size)


def apply_rotary_emb(hidden_states, rotary_emb):
    """The H3 rotary embedding is defined by diffusers; use its function like the reference."""
    try:
        from diffusers.models.transformers.transformer_minimax_h3 import _apply_rotary_emb
    except ImportError as error:
        raise ImportError("rotary embeddings for MiniMax-H3 need diffusers' transformer_minimax_h3") from error
    return _apply_rotary_emb(hidden_states, *rotary_emb)


def _sol_attention(controller, q, k, v, layout, layer, *, return_bthd=False, inputs_bthd=False):
    """q, k, v as BHTD (inputs_bthd=False) or BTHD; returns BTHD when return_bthd.

    A controller with a head_budget_allocator gets per-head Top-K budgets for this layer
    from allocator(layer, evaluation_index, V as BHTD, video_tokens) (processor.py:782-796)."""
    cfg = controller.config
    allocator = getattr(controller, "head_budget_allocator", None)
    if allocator is not None:
        if cfg.sol_route_topk_ratio is None:
            raise ValueError("head budget allocation requires a Top-K configuration")
        budget_values = v.permute(0, 2, 1, 3) if inputs_bthd else v
        controller.head_topk_budget = allocator(layer, controller.evaluation_index, budget_values,
                                                layout.video_tokens)
    else:
        controller.head_topk_budget = None
    if not inputs_bthd:
        q, k, v = (x.permute(0, 2, 1, 3).contiguous() for x in (q, k, v))
    return spark_attention_bthd(controller, q, k, v, layout, layer, return_bthd=return_bthd)


class _H3SparseProcessor:
    def __init__(self, layer: int, original, controller: _Controller):
        self.layer = layer
        self.original = original
        self.controller = controller

    def _dense(self, attn, hidden_states, rotary_emb, attention_mask, reason: str):
        self.controller.counts[f"dense:{reason}"] += 1
        return self.original(attn, hidden_states, rotary_emb, attention_mask)

    def __call__(self, attn, hidden_states, rotary_emb=None, attention_mask=None):
        c = self.controller
        cfg = c.config
        layout = c.layout
        if c.is_warmup:
            return self._dense(attn, hidden_states, rotary_emb, attention_mask, "warmup")
        if c.evaluation_index in cfg.sol_extra_dense_evaluations:
            return self._dense(attn, hidden_states, rotary_emb, attention_mask, "extra_dense_evaluation")
        if self.layer < cfg.sol_dense_layers:
            return self._dense(attn, hidden_states, rotary_emb, attention_mask, "dense_layer")
        if self.layer in cfg.sol_extra_dense_layers:
            return self._dense(attn, hidden_states, rotary_emb, attention_mask, "extra_dense_layer")
        if hidden_states.shape[1] < cfg.sol_min_tokens:
            return self._dense(attn, hidden_states, rotary_emb, attention_mask, "short_sequence")
        if layout is None:
            raise RuntimeError("sparse H3 processor did not receive packed-layout metadata")
        if attention_mask is not None:
            raise RuntimeError("sparse H3 processor does not accept an external attention mask")
        if hidden_states.shape[0] != 1:
            raise RuntimeError("official sparse kernels currently require packed H3 batch size 1")
        if hidden_states.shape[1] != layout.sequence_length:
            raise RuntimeError("packed layout length does not match H3 hidden states: "
                               f"{layout.sequence_length} != {hidden_states.shape[1]}")
        query, key, value = self._project(attn, hidden_states, rotary_emb)
        dtype = query.dtype
        permutation = layout.permutation
        # Packed BTHD (video first); the B200 kernels consume it directly.
        packed_q = query.index_select(1, permutation).contiguous()
        del query
        packed_k = key.index_select(1, permutation).contiguous()
        del key
        packed_v = value.index_select(1, permutation).contiguous()
        del value
        output = _sol_attention(c, packed_q, packed_k, packed_v, layout, self.layer, return_bthd=True,
                                inputs_bthd=True)
        output = output.index_select(1, layout.inverse_permutation).flatten(2, 3).to(dtype)
        output = attn.to_out[0](output)
        output = attn.to_out[1](output)
        c.counts["sparse:sol"] += 1
        return output

    @staticmethod
    def _project(attn, hidden_states, rotary_emb):
        """Q/K/V projections, per-head norms and rotary embedding (processor.py:896-933)."""
        if getattr(attn, "fused_projections", False):
            query, key, value = attn.to_qkv(hidden_states).chunk(3, dim=-1)
        elif hasattr(attn.to_q, "forward_quantized"):
            from .fp8_linear import forward_qkv_shared
            query, key, value = forward_qkv_shared(attn, hidden_states)
        else:
            query, key, value = attn.to_q(hidden_states), attn.to_k(hidden_states), attn.to_v(hidden_states)
        query = attn.norm_q(query.unflatten(-1, (attn.heads, -1)))
        key = attn.norm_k(key.unflatten(-1, (attn.heads, -1)))
        value = value.unflatten(-1, (attn.heads, -1))
        if rotary_emb is not None:
            query = apply_rotary_emb(query, rotary_emb)
            key = apply_rotary_emb(key, rotary_emb)
        return query, key, value


class H3SparseAttentionPlugin:
    """Context-managed, reversible processor installation on one H3 transformer."""

    def __init__(self, transformer, config: H3SparseAttentionConfig):
        self.transformer = transformer
        self.config = config
        self.controller = _Controller(config)
        self._originals: list[tuple[Any, Any]] = []
        self._hook = None
        self._active = False

    def __enter__(self) -> "H3SparseAttentionPlugin":
        if self._active:
            raise RuntimeError("plugin is already active")
        self.controller.reset()
        blocks = getattr(self.transformer, "transformer_blocks", None)
        if blocks is None:
            raise TypeError("expected a MiniMax-H3 transformer with transformer_blocks")
        try:
            self._hook = self.transformer.register_forward_pre_hook(self.controller.begin_forward, with_kwargs=True)
            for layer, block in enumerate(blocks):
                attn = block["attn"] if isinstance(block, torch.nn.ModuleDict) else block.attn
                original = attn.get_processor()
                self._originals.append((attn, original))
                attn.set_processor(_H3SparseProcessor(layer, original, self.controller))
            self._active = True
            return self
        except Exception:
            self.remove()
            raise

    def reset(self) -> None:
        self.controller.reset()

    def summary(self) -> dict[str, Any]:
        return self.controller.summary()

    def remove(self) -> None:
        for attn, original in reversed(self._originals):
            attn.set_processor(original)
        self._originals.clear()
        if self._hook is not None:
            self._hook.remove()
            self._hook = None
        self.controller.layout = None
        self.controller.rope_sol_key_clustering_static.clear()
        self.controller._virtual_query_layout_cache.clear()
        self.controller.landmark_reblock_hierarchy = None
        self._active = False

    def __exit__(self, exc_type, exc_value, traceback) -> bool:
        self.remove()
        return False


def install_h3_sparse_attention(transformer, config: H3SparseAttentionConfig) -> H3SparseAttentionPlugin:
    return H3SparseAttentionPlugin(transformer, config)


def _fold_installer_args(overrides, *, dense_layers, min_tokens, warmup_mode, warmup_ratio, warmup_steps,
                         topk_ratio=None):
    if dense_layers is not None:
        if "sol_dense_layers" in overrides:
            raise ValueError("dense_layers cannot be combined with legacy sol_dense_layers")
        if type(dense_layers) is not int or dense_layers < 0:
            raise ValueError("dense_layers must be a nonnegative integer")
        overrides["sol_dense_layers"] = dense_layers
    if min_tokens is not None:
        if "sol_min_tokens" in overrides:
            raise ValueError("min_tokens cannot be combined with legacy sol_min_tokens")
        if type(min_tokens) is not int or min_tokens < 0:
            raise ValueError("min_tokens must be a nonnegative integer")
        overrides["sol_min_tokens"] = min_tokens
    if topk_ratio is not None:
        if "sol_route_topk_ratio" in overrides:
            raise ValueError("topk_ratio cannot be combined with legacy sol_route_topk_ratio")
        overrides["sol_route_topk_ratio"] = topk_ratio
    for name, value in (("warmup_mode", warmup_mode), ("warmup_ratio", warmup_ratio), ("warmup_steps", warmup_steps)):
        if value is not None:
            overrides[name] = value
    return overrides


def install_h3_sol_attn(transformer, num_inference_steps=None, *, num_denoise_steps=None, warmup_mode=None,
                        warmup_ratio=None, warmup_steps=None, dense_layers=None, min_tokens=None,
                        **config_overrides) -> H3SparseAttentionPlugin:
    """Sol-policy plugin (processor.py:1047-1089); its sparse path needs Top-K routing here."""
    overrides = _fold_installer_args(config_overrides, dense_layers=dense_layers, min_tokens=min_tokens,
                                     warmup_mode=warmup_mode, warmup_ratio=warmup_ratio, warmup_steps=warmup_steps)
    return install_h3_sparse_attention(
        transformer, H3SparseAttentionConfig.sol(num_inference_steps, num_denoise_steps=num_denoise_steps, **overrides))


def install_h3_spark_attn(transformer, num_inference_steps=None, *, num_denoise_steps=None, warmup_mode=None,
                          warmup_ratio=None, warmup_steps=None, dense_layers=None, min_tokens=None, topk_ratio=None,
                          mode="full", **config_overrides) -> H3SparseAttentionPlugin:
    """The Spark plugin: Top-K routing, global-anchor reweighting, optional LMv2 reblocking
    (processor.py:1092-1144)."""
    overrides = _fold_installer_args(config_overrides, dense_layers=dense_layers, min_tokens=min_tokens,
                                     warmup_mode=warmup_mode, warmup_ratio=warmup_ratio, warmup_steps=warmup_steps,
                                     topk_ratio=topk_ratio)
    return install_h3_sparse_attention(
        transformer, H3SparseAttentionConfig.spark(num_inference_steps, num_denoise_steps=num_denoise_steps,
                                                   mode=mode, **overrides))
