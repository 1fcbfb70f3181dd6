"""Failure detection on the GPU without a fault: a bounded wait that nothing satisfies gives
up, raises the CTA abort flag (which releases the CTA's other waits) and reports its site
code through the device status word; the context stays usable afterwards."""
import numpy as np
import pytest
import torch

from oracle import oracle
from spark_h3_b200 import _lib, ops
from spark_h3_b200.synthetic import make_qkv

pytestmark = pytest.mark.gpu

SELFTEST_WAIT_SITE = 990  # SB_SELFTEST_WAIT_SITE in include/spark_h3_b200.h


def test_bounded_wait_times_out_and_context_stays_usable(cuda_device):
    dev = cuda_device
    assert ops.read_device_status(dev) == 0
    result = torch.full((4,), -1, dtype=torch.int32, device=dev)
    with torch.cuda.device(dev):
        _lib.call("sb_selftest_wait_timeout", 1_000_000, result.data_ptr(), ops._stream(dev))
    assert ops.read_device_status(dev) == SELFTEST_WAIT_SITE
    # warp 0 timed out, warp 1 was released by the abort flag; both left in bounded time
    assert result.tolist() == [0, 1, 0, 1]
    assert ops.read_device_status(dev) == 0  # reading clears the word

    # The context is still usable: a small layer runs and matches the oracle.
    q, k, v = make_qkv((2, 16, 40), 2, 128, seed=1, dtype=torch.bfloat16, q_scale=128 ** -0.5)
    out = ops.spark_layer(q.to(dev), k.to(dev), v.to(dev), block=128, topk_ratio=0.1)
    torch.cuda.synchronize()
    assert ops.read_device_status(dev) == 0
    host = lambda t: oracle.Tensor(t.cpu().contiguous().view(torch.int16).numpy().view(np.uint16), "bfloat16")
    ref = oracle.spark_layer(host(q), host(k), host(v), block=128, topk_ratio=0.1)
    assert np.abs(out.float().cpu().numpy() - ref["out"]).max() <= 2e-2
