"""The streamed layer (pinned host tensors, head chunks, overlapped copies) against the
device-resident layer: every stage is per (batch, head), so the results are identical."""
from __future__ import annotations

import pytest
import torch

from spark_h3_b200 import ops
from spark_h3_b200.synthetic import make_qkv

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("grid,heads,chunks,block,dtype", [((2, 24, 40), 8, 4, 128, torch.bfloat16),
                                                           ((3, 16, 21), 4, 2, 64, torch.bfloat16),
                                                           ((2, 16, 16), 4, 4, 64, torch.float32)])
def test_streamed_matches_device_layer(cuda_device, grid, heads, chunks, block, dtype):
    D = 128 if dtype == torch.bfloat16 else 64
    q, k, v = make_qkv(grid, heads, D, seed=3, dtype=dtype, q_scale=D ** -0.5, device=cuda_device)
    T = q.shape[1]
    video = T - 7  # a context suffix past the video tokens
    expected = ops.spark_layer(q, k, v, block=block, topk_ratio=0.2, video_tokens=video)
    hq, hk, hv = (t.cpu().pin_memory() for t in (q, k, v))
    out = torch.empty(hq.shape, dtype=dtype, pin_memory=True)
    for _ in range(2):  # twice: the second call reuses nothing from the first
        out.zero_()
        ops.spark_layer_streamed(hq, hk, hv, out, chunks=chunks, block=block, topk_ratio=0.2, video_tokens=video)
        torch.cuda.current_stream().synchronize()
        assert torch.equal(out, expected.cpu())


def test_streamed_rejects_device_or_unpinned_tensors(cuda_device):
    x = torch.zeros(1, 128, 4, 128, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="pinned"):
        ops.spark_layer_streamed(x, x, x, x)
    p = x.pin_memory()
    with pytest.raises(ValueError, match="chunks"):
        ops.spark_layer_streamed(p, p, p, p, chunks=3)
