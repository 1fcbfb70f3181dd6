"""Processor gates and plugin installation on CPU (no kernel launches)."""
import pytest
import torch

from spark_h3_b200 import H3SparseAttentionConfig, install_h3_spark_attn
from spark_h3_b200.processor import _Controller, _H3SparseProcessor


class FakeAttention(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.processor = "original-processor"

    def get_processor(self):
        return self.processor

    def set_processor(self, processor):
        self.processor = processor


class FakeBlock(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.attn = FakeAttention()


class FakeTransformer(torch.nn.Module):
    def __init__(self, layers=2):
        super().__init__()
        self.transformer_blocks = torch.nn.ModuleList([FakeBlock() for _ in range(layers)])

    def forward(self, hidden_states, token_tags=None, position_ids=None):
        return hidden_states


def test_short_sequences_stay_dense_and_missing_layout_is_an_error():
    cfg = H3SparseAttentionConfig.spark(num_denoise_steps=1, warmup_mode="warmup_steps", warmup_steps=0)
    controller = _Controller(cfg)
    controller.evaluation_index = 0
    marker = object()
    processor = _H3SparseProcessor(0, lambda attn, hs, rot, mask: marker, controller)
    assert processor(None, torch.empty(1, 8191, 1)) is marker
    assert controller.counts["dense:short_sequence"] == 1
    with pytest.raises(RuntimeError, match="packed-layout metadata"):
        processor(None, torch.empty(1, 8192, 1))


def test_warmup_and_dense_layers_use_the_original_processor():
    cfg = H3SparseAttentionConfig.spark(num_denoise_steps=3, warmup_mode="warmup_steps", warmup_steps=1,
                                        sol_dense_layers=1, sol_min_tokens=0)
    controller = _Controller(cfg)
    calls = []
    original = lambda attn, hs, rot, mask: calls.append(hs.shape) or "dense"
    controller.evaluation_index = 0
    assert _H3SparseProcessor(3, original, controller)(None, torch.empty(1, 4, 1)) == "dense"
    assert controller.counts["dense:warmup"] == 1
    controller.evaluation_index = 1
    assert _H3SparseProcessor(0, original, controller)(None, torch.empty(1, 4, 1)) == "dense"
    assert controller.counts["dense:dense_layer"] == 1


def test_plugin_installs_hooks_and_restores_processors():
    model = FakeTransformer()
    plugin = install_h3_spark_attn(model, num_denoise_steps=2, mode="reweight_only")
    with plugin:
        assert all(isinstance(b.attn.processor, _H3SparseProcessor) for b in model.transformer_blocks)
        tags = torch.zeros(8, dtype=torch.long)
        pos = torch.cartesian_prod(torch.arange(2), torch.arange(2), torch.arange(2))
        model(torch.zeros(1, 8, 4), token_tags=tags, position_ids=pos)
        assert plugin.controller.layout.video_tokens == 8 and plugin.summary()["completed_evaluations"] == 1
        model(torch.zeros(1, 8, 4), token_tags=tags, position_ids=pos)
        with pytest.raises(RuntimeError, match="more transformer evaluations"):
            model(torch.zeros(1, 8, 4), token_tags=tags, position_ids=pos)
    assert all(b.attn.processor == "original-processor" for b in model.transformer_blocks)
    assert not model._forward_pre_hooks


def test_plugin_restores_processors_when_the_body_raises():
    model = FakeTransformer()
    with pytest.raises(ValueError, match="boom"):
        with install_h3_spark_attn(model, num_denoise_steps=2):
            raise ValueError("boom")
    assert all(b.attn.processor == "original-processor" for b in model.transformer_blocks)
    assert not model._forward_pre_hooks


def test_forward_without_layout_metadata_is_rejected():
    model = FakeTransformer()
    with install_h3_spark_attn(model, num_denoise_steps=2):
        with pytest.raises(RuntimeError, match="token_tags/position_ids"):
            model(torch.zeros(1, 8, 4))


def test_sparse_query_prefix_by_tail_mode():
    # spark_integration.py:72-91 and the reference's own expectations
    # (tests/test_global_reweight_followup.py:14-16).
    from spark_h3_b200.ops import sparse_query_tokens

    assert sparse_query_tokens(8329, 8193, 64, "dense") == 8192
    assert sparse_query_tokens(8329, 8193, 64, "pad") == 8256
    assert sparse_query_tokens(8329, 8193, 128, "pad") == 8320
    with pytest.raises(ValueError, match="too short to pad"):
        sparse_query_tokens(8200, 8193, 64, "pad")
    with pytest.raises(ValueError, match="tail_mode"):
        sparse_query_tokens(8329, 8193, 64, "wrap")


def test_query_prefix_off_a_block_boundary_is_rejected():
    # tests/test_global_reweight_followup.py:66-67: a sparse query prefix that does not end
    # on a query block is a ValueError, raised before any device work.
    from spark_h3_b200 import ops

    q = torch.zeros(1, 8329, 1, 128, dtype=torch.bfloat16)
    for bad in (8191, 8193, -64, 8384):
        with pytest.raises(ValueError, match="query-block boundary"):
            ops.sparse_attention(q, q, q, 64, None, None, None, None, query_tokens=bad, sink_first=0,
                                 sink_last=0)
        with pytest.raises(ValueError, match="query-block boundary"):
            ops.tail_merge(q, None, None, None, None, q, None, block=64, entry_tokens=64, group_tokens=64,
                           query_tokens=bad, sink_first=0, sink_last=0)


def test_oracle_pad_fill_is_the_tail_mean():
    # The rows that pad the final video block hold the fp32 mean of its video rows rounded to
    # bf16, as q[:, tail:video].mean(1, dtype=float32).to(bf16) (spark_integration.py:1180-1187).
    import numpy as np

    from oracle import oracle

    torch.manual_seed(5)
    q = torch.randn(1, 137, 2, 128).to(torch.bfloat16)
    video, block = 97, 64
    host = oracle.Tensor(q.view(torch.int16).numpy().view(np.uint16), "bfloat16")
    padded = oracle.padded_tail(host, video, 128, block)
    expected = q[:, 64:video].mean(1, keepdim=True, dtype=torch.float32).to(torch.bfloat16)
    got = torch.from_numpy(padded.data.view(np.int16)).view(torch.bfloat16)
    assert torch.equal(got[:, video:128], expected.expand(-1, 128 - video, -1, -1))
    assert torch.equal(got[:, :video], q[:, :video]) and torch.equal(got[:, 128:], q[:, 128:])


def test_head_budget_allocator_sets_the_layer_budget(monkeypatch):
    """processor.py:782-796: a controller's head_budget_allocator is called per sparse layer
    with (layer, evaluation, V as BHTD, video tokens), and its result reaches the attention
    seam as controller.head_topk_budget; without one the budget is cleared."""
    from spark_h3_b200 import processor as proc

    cfg = H3SparseAttentionConfig.spark(num_denoise_steps=1, warmup_mode="warmup_steps", warmup_steps=0)
    controller = _Controller(cfg)
    controller.evaluation_index = 0
    seen = {}

    def fake_seam(ctrl, q, k, v, layout, layer, return_bthd=True):
        seen["budget"] = ctrl.head_topk_budget
        return q

    monkeypatch.setattr(proc, "spark_attention_bthd", fake_seam)
    calls = []

    def allocator(layer, evaluation, values, video_tokens):
        calls.append((layer, evaluation, tuple(values.shape), video_tokens))
        return torch.tensor([1, 2])

    controller.head_budget_allocator = allocator
    q = torch.zeros(1, 8, 2, 4)  # BTHD
    layout = type("L", (), dict(video_tokens=6))()
    proc._sol_attention(controller, q, q, q, layout, 3, return_bthd=True, inputs_bthd=True)
    assert calls == [(3, 0, (1, 2, 8, 4), 6)]
    assert seen["budget"].tolist() == [1, 2]
    controller.head_budget_allocator = None
    proc._sol_attention(controller, q, q, q, layout, 3, return_bthd=True, inputs_bthd=True)
    assert seen["budget"] is None


def test_head_budget_needs_one_budget_per_head():
    from spark_h3_b200.attention import _head_budgets

    assert _head_budgets(None, 4, torch.device("cpu")) is None
    assert _head_budgets([1, 2, 3, 4], 4, torch.device("cpu")).dtype == torch.int32
    with pytest.raises(ValueError, match="expected one budget per head"):
        _head_budgets(torch.tensor([1, 2, 3]), 4, torch.device("cpu"))


def test_legacy_full_query_prefix():
    """sol_legacy_full_query (spark_integration.py:925-933): the sparse prefix covers every video
    block, the partial final one included; a final block the sequence does not fill is refused."""
    from spark_h3_b200.ops import sparse_query_tokens

    assert sparse_query_tokens(2262, 2100, 64, "legacy_full") == 2112
    assert sparse_query_tokens(2262, 2048, 64, "legacy_full") == 2048
    assert sparse_query_tokens(2262, 2100, 128, "legacy_full") == 2176
    with pytest.raises(NotImplementedError):
        sparse_query_tokens(2105, 2100, 64, "legacy_full")
