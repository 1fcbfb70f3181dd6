"""CUDA-graph capture of a whole Spark layer (pool, anchor, summaries, route, attention, tail
merge and dense rows): no host synchronisation and no allocation outside torch's graph pool,
so a replay after Q changes in place matches an eager run bit for bit.  The reference pins
the same property for its fused layer (tests/test_global_reweight_followup.py:60-65)."""
import pytest
import torch

from spark_h3_b200 import ops
from spark_h3_b200.synthetic import make_qkv

pytestmark = pytest.mark.gpu


def _inputs(device):
    # 1,584 video tokens (a partial final block at 64 and 128) followed by 150 context tokens.
    q, k, v = make_qkv((3, 16, 33), 2, 128, seed=41, dtype=torch.bfloat16, q_scale=128 ** -0.5)
    extra = make_qkv((1, 10, 15), 2, 128, seed=42, dtype=torch.bfloat16, q_scale=128 ** -0.5)
    q, k, v = (torch.cat((a, b), dim=1).to(device) for a, b in zip((q, k, v), extra))
    return q, k, v, 3 * 16 * 33


@pytest.mark.parametrize("block,tail_mode,granularity", [(128, "dense", "query"), (64, "pad", "query"),
                                                         (64, "dense", "block8x8"), (128, "pad", "block")])
def test_spark_layer_replays_in_cuda_graph(cuda_device, block, tail_mode, granularity):
    q, k, v, video = _inputs(cuda_device)
    kwargs = dict(block=block, topk_ratio=0.1, video_tokens=video, tail_mode=tail_mode,
                  tail_granularity=granularity)
    eager = ops.spark_layer(q, k, v, **kwargs).clone()
    side = torch.cuda.Stream(cuda_device)
    side.wait_stream(torch.cuda.current_stream(cuda_device))
    with torch.cuda.stream(side):
        ops.spark_layer(q, k, v, **kwargs)
    torch.cuda.current_stream(cuda_device).wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        captured = ops.spark_layer(q, k, v, **kwargs)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(captured, eager)
    q.mul_(0.5)
    graph.replay()
    expected = ops.spark_layer(q, k, v, **kwargs)
    torch.cuda.synchronize()
    assert not torch.equal(expected, eager)
    assert torch.equal(captured, expected)
    assert ops.read_device_status(cuda_device) == 0
    del graph
