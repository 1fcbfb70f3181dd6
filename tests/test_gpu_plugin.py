"""The installed plugin end to end on the GPU: projections, packed layout, Spark attention
through libsparkh3b200.so and the inverse permutation, against the CPU oracle."""
import numpy as np
import pytest
import torch

from oracle import oracle
from spark_h3_b200 import install_h3_spark_attn

pytestmark = pytest.mark.gpu


class TinyAttention(torch.nn.Module):
    """The attribute surface the processor reads from a MiniMax-H3 attention module."""

    def __init__(self, hidden=256, heads=2):
        super().__init__()
        self.heads = heads
        self.fused_projections = False
        self.to_q = torch.nn.Linear(hidden, hidden, bias=False)
        self.to_k = torch.nn.Linear(hidden, hidden, bias=False)
        self.to_v = torch.nn.Linear(hidden, hidden, bias=False)
        self.norm_q = torch.nn.Identity()
        self.norm_k = torch.nn.Identity()
        self.to_out = torch.nn.ModuleList([torch.nn.Identity(), torch.nn.Identity()])
        self.processor = None

    def get_processor(self):
        return self.processor

    def set_processor(self, processor):
        self.processor = processor

    def forward(self, hidden_states):
        return self.processor(self, hidden_states)


class TinyTransformer(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.transformer_blocks = torch.nn.ModuleList([torch.nn.Module()])
        self.transformer_blocks[0].attn = TinyAttention()

    def forward(self, hidden_states, token_tags=None, position_ids=None):
        return self.transformer_blocks[0].attn(hidden_states)


def host(t):
    t = t.detach().cpu().contiguous()
    return oracle.Tensor(t.view(torch.int16).numpy().view(np.uint16), "bfloat16")


@pytest.mark.parametrize("mode,block,tail_mode", [("reweight_only", 64, "dense"), ("topk_only", 64, "dense"),
                                                  ("reweight_only", 128, "dense"), ("reweight_only", 64, "pad"),
                                                  ("reweight_only", 128, "pad")])
def test_plugin_matches_oracle(cuda_device, mode, block, tail_mode):
    torch.manual_seed(3)
    dev = cuda_device
    model = TinyTransformer().to(dev, torch.bfloat16)
    for lin in (model.transformer_blocks[0].attn.to_q, model.transformer_blocks[0].attn.to_k,
                model.transformer_blocks[0].attn.to_v):
        torch.nn.init.normal_(lin.weight, std=0.06)
    grid = (2, 16, 40) if tail_mode == "dense" else (2, 16, 41)  # pad: a partial final video block
    video = grid[0] * grid[1] * grid[2]
    text = 50 if tail_mode == "dense" else 100
    tags = torch.cat([torch.ones(text), torch.zeros(video)]).long()     # text first in the raw order
    pos = torch.cat([torch.zeros(text, 3, dtype=torch.long),
                     torch.cartesian_prod(*(torch.arange(n) for n in grid))])
    x = torch.randn(1, video + text, 256, dtype=torch.bfloat16).to(dev)
    attn = model.transformer_blocks[0].attn
    with install_h3_spark_attn(model, num_denoise_steps=1, warmup_mode="warmup_steps", warmup_steps=0,
                               min_tokens=0, mode=mode, sol_block_size=block,
                               sol_video_tail_mode=tail_mode) as plugin:
        out = model(x, token_tags=tags.to(dev), position_ids=pos.to(dev))
        layout = plugin.controller.layout
        summary = plugin.summary()
    torch.cuda.synchronize()
    assert summary["processor_calls"]["sparse:sol"] == 1
    assert summary["sol_backend"] == "b200_sm100_fused_virtual_query"
    # Expected: same projections, packed order, oracle attention, inverse order.
    with torch.no_grad():
        q = attn.to_q(x).unflatten(-1, (2, -1)).index_select(1, layout.permutation)
        k = attn.to_k(x).unflatten(-1, (2, -1)).index_select(1, layout.permutation)
        v = attn.to_v(x).unflatten(-1, (2, -1)).index_select(1, layout.permutation)
    weighted = mode != "topk_only"
    ref = oracle.spark_layer(host(q), host(k), host(v), block=block, topk_ratio=0.1, video_tokens=video,
                             weighted_kv=weighted, mass_bias=weighted, tail_mode=tail_mode)
    expected = torch.from_numpy(ref["out"]).to(dev)[:, layout.inverse_permutation].flatten(2, 3)
    err = (out.float() - expected).abs().max().item()
    cos = torch.nn.functional.cosine_similarity(out.float().flatten(), expected.flatten(), dim=0).item()
    assert err <= 2e-2 and cos >= 0.9995, (err, cos)
