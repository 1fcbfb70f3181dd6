"""H3SparseAttentionConfig and the installers: defaults, presets and the validation errors
callers of the reference rely on (h3_sparse_attention/processor.py:40-535, 1092-1144)."""
import inspect

import pytest

from spark_h3_b200 import H3SparseAttentionConfig, install_h3_sol_attn, install_h3_spark_attn


def test_spark_defaults():
    cfg = install_h3_spark_attn(object(), num_denoise_steps=19).config
    assert cfg.method == "sol" and cfg.total_evaluations == 19
    assert cfg.sol_route_topk_ratio == 0.1 and cfg.sol_route_topk_cutoff_mode == "gemm_radix"
    assert cfg.sol_route_topk_execution == "packed_external_no_route_qk"
    assert cfg.sol_min_tokens == 8192 and cfg.sol_dense_layers == 0
    assert cfg.sol_global_anchor_dtype == "bfloat16" and cfg.sol_spark_mode == "full"
    assert cfg.sol_reweight_components == "full" and cfg.sol_video_tail_mode == "dense"
    assert cfg.sol_landmark_preprocess and cfg.sol_landmark_preprocess_version == "v2"
    assert cfg.sol_virtual_query_levels_up == 99 and cfg.sol_virtual_query_target_blocks is None
    assert not cfg.sol_local_blocks_enabled and cfg.sol_local_block_radius == -1
    assert cfg.landmark_tree_v2_children == 16 and cfg.landmark_tree_v2_landmark_count == 32
    assert cfg.sol_block_size == 64


def test_denoise_step_counts():
    assert H3SparseAttentionConfig.spark(num_denoise_steps=8).total_evaluations == 8
    assert H3SparseAttentionConfig.spark(num_inference_steps=20).total_evaluations == 19
    assert H3SparseAttentionConfig.sol(num_inference_steps=50).total_evaluations == 49
    assert H3SparseAttentionConfig().total_evaluations == 19
    with pytest.raises(ValueError, match="either num_denoise_steps or num_inference_steps"):
        H3SparseAttentionConfig.spark(num_inference_steps=20, num_denoise_steps=19)
    with pytest.raises(ValueError, match="num_denoise_steps"):
        H3SparseAttentionConfig.spark(num_denoise_steps=0)


def test_warmup_and_installer_arguments():
    params = inspect.signature(install_h3_spark_attn).parameters
    for name in ("warmup_mode", "warmup_ratio", "warmup_steps", "dense_layers", "min_tokens", "topk_ratio", "mode"):
        assert name in params
    assert H3SparseAttentionConfig.spark(num_denoise_steps=19).dense_evaluations == 4
    assert H3SparseAttentionConfig.spark(num_denoise_steps=8, warmup_ratio=0.25).dense_evaluations == 2
    assert H3SparseAttentionConfig.spark(num_denoise_steps=3, warmup_mode="warmup_steps",
                                         warmup_steps=4).dense_evaluations == 3
    assert H3SparseAttentionConfig.spark(num_denoise_steps=5, warmup_percent=20).dense_evaluations == 1
    plugin = install_h3_spark_attn(object(), num_denoise_steps=19, warmup_mode="warmup_steps", warmup_steps=4)
    assert plugin.summary()["warmup_mode"] == "warmup_steps" and plugin.summary()["warmup_steps"] == 4
    assert install_h3_spark_attn(object(), sol_dense_layers=2).config.sol_dense_layers == 2
    assert install_h3_spark_attn(object(), topk_ratio=0.2).config.sol_route_topk_ratio == 0.2
    assert install_h3_spark_attn(object(), min_tokens=0).config.sol_min_tokens == 0
    for kwargs, pattern in [(dict(dense_layers=1, sol_dense_layers=1), "cannot be combined"),
                            (dict(dense_layers=-1), "dense_layers"),
                            (dict(min_tokens=8192, sol_min_tokens=8192), "cannot be combined"),
                            (dict(min_tokens=-1), "min_tokens"),
                            (dict(topk_ratio=0.1, sol_route_topk_ratio=0.1), "cannot be combined"),
                            (dict(topk_ratio=0.0), "sol_route_topk_ratio")]:
        with pytest.raises(ValueError, match=pattern):
            install_h3_spark_attn(object(), **kwargs)
    with pytest.raises(ValueError, match="warmup_percent cannot be combined"):
        H3SparseAttentionConfig.spark(warmup_percent=20, warmup_mode="warmup_steps", warmup_steps=4)
    for kwargs, pattern in [(dict(warmup_mode="invalid"), "warmup_mode"), (dict(warmup_ratio=1.1), "warmup_ratio"),
                            (dict(warmup_steps=-1), "warmup_steps")]:
        with pytest.raises(ValueError, match=pattern):
            H3SparseAttentionConfig.spark(**kwargs)


def test_modes_and_disabled_options():
    for mode, (reblock, reweight) in {"topk_only": (False, False), "reblock_only": (True, False),
                                      "reweight_only": (False, True), "full": (True, True)}.items():
        cfg = H3SparseAttentionConfig.spark(20, mode=mode)
        assert cfg.sol_landmark_preprocess is reblock
        assert (cfg.sol_reweight_components != "none") is reweight
    assert H3SparseAttentionConfig.spark(20, mode="topk_only").sol_local_blocks_enabled
    assert H3SparseAttentionConfig.sol(20).sol_local_blocks_enabled
    with pytest.raises(ValueError, match="threshold.*disabled"):
        H3SparseAttentionConfig.spark(20, sol_route_topk_execution="threshold")
    with pytest.raises(ValueError, match="fused.*disabled"):
        H3SparseAttentionConfig.spark(20, landmark_tree_v2_midpoint_direction_mode="fused")
    with pytest.raises(ValueError, match="mode must be"):
        H3SparseAttentionConfig.spark(20, mode="invalid")
    with pytest.raises(ValueError, match="requires Top-K or virtual-query"):
        H3SparseAttentionConfig.sol(20, sol_video_tail_mode="pad")
    for legacy in ({"sol_virtual_query_levels_up": 2}, {"sol_landmark_preprocess": False}):
        with pytest.raises(ValueError, match="public Spark modes"):
            H3SparseAttentionConfig.spark(20, **legacy)
    with pytest.raises(ValueError, match="sol_sparse_video_scope"):
        H3SparseAttentionConfig.spark(20, sol_sparse_video_scope="all")
    with pytest.raises(ValueError, match="Spark component modes require Top-K routing"):
        H3SparseAttentionConfig.spark(3, sol_route_topk_ratio=None)


def test_exact_block_radius():
    cfg = H3SparseAttentionConfig.sol(20, sol_route_topk_ratio=0.1, sol_exact_block_radius=0)
    assert cfg.sol_local_blocks_enabled and cfg.sol_local_block_radius == 0 and cfg.kernel_local_radius == 0
    assert H3SparseAttentionConfig.spark(20, mode="topk_only").kernel_local_radius == -1
    with pytest.raises(ValueError, match="requires Top-K routing"):
        H3SparseAttentionConfig.sol(20, sol_exact_block_radius=0)
    with pytest.raises(ValueError, match="requires landmark_tree_v2_layout_reuse"):
        H3SparseAttentionConfig.spark(20, sol_exact_block_radius=0)
    with pytest.raises(ValueError, match="not both"):
        H3SparseAttentionConfig.sol(20, sol_route_topk_ratio=0.1, sol_exact_block_radius=0,
                                    sol_force_local_blocks=False)
    assert H3SparseAttentionConfig.spark(20, sol_exact_block_radius=2,
                                         landmark_tree_v2_layout_reuse="q_from_k").sol_local_block_radius == 2


def test_block_size_extension():
    assert H3SparseAttentionConfig.spark(20, sol_block_size=128).sol_block_size == 128
    with pytest.raises(ValueError, match="sol_block_size"):
        H3SparseAttentionConfig.spark(20, sol_block_size=96)
    assert install_h3_sol_attn(object(), num_denoise_steps=9).config.total_evaluations == 9
