"""The allocation-free route entry point, sb_route_topk_noalloc, against sb_route_topk.

Callers that cannot hand the library a device workspace (a host binding only this C ABI
through a thin FFI with no device allocator, or a loop that cannot afford the device
synchronisation of cudaMalloc) use the variant whose score scratch is a fixed file-scope
device array.  Both are called here through the C ABI on the same inputs; the route is
integer output, so the comparison is exact, and the variant is called twice in a row to show
that the shared scratch left by one call does not leak into the next.

This file is named to be collected last, so a run that stops at the first failure has
already run every other test.
"""
import ctypes
import math

import pytest
import torch

from spark_h3_b200 import _lib, ops
from spark_h3_b200.synthetic import make_qkv

pytestmark = pytest.mark.gpu


def _noalloc(lib, qc, kc, QB, candidates, topk, packed, indices, stream):
    B, NB, H, D = qc.shape
    return lib.sb_route_topk_noalloc(qc.data_ptr(), kc.data_ptr(), _lib.BF16, B, QB, NB, H, D, candidates, topk,
                                     ops.scale_log2(D), packed.data_ptr(), indices.data_ptr(), stream)


@pytest.mark.parametrize("grid,heads,block", [((4, 16, 33), 2, 128), ((8, 40, 160), 8, 64)])
def test_noalloc_route_equals_workspace_route(cuda_device, grid, heads, block):
    # The second case has 8 heads x 800 candidate blocks x 800 query blocks = 5.1M scores,
    # more than the 4M-float scratch, so the variant works through two chunks.
    dev = cuda_device
    q, k, v = make_qkv(grid, heads, 128, seed=9, device=dev, dtype=torch.bfloat16, q_scale=128 ** -0.5)
    T = q.shape[1]
    qb = T // block
    nb = math.ceil(T / block)
    topk = ops.target_topk(0.1, qb)
    qc = ops.pool_queries(q, block)
    kc, _, _, _ = ops.pool_keys_summaries(k, None, None, block, want_summaries=False)
    lib = _lib.load()
    stream = torch.cuda.current_stream(dev).cuda_stream

    words = math.ceil(nb / 32)
    ref_packed = torch.empty((1, qb, heads, words), device=dev, dtype=torch.int32)
    ref_idx = torch.empty((1, qb, heads, topk), device=dev, dtype=torch.int32)
    workspace = torch.empty(lib.sb_route_workspace_bytes(1, qb, heads, qb), device=dev, dtype=torch.uint8)
    rc = lib.sb_route_topk(qc.data_ptr(), kc.data_ptr(), _lib.BF16, 1, qb, nb, heads, 128, qb, topk,
                           ops.scale_log2(128), workspace.data_ptr(), ref_packed.data_ptr(), ref_idx.data_ptr(),
                           stream)
    assert rc == 0, lib.sb_last_error()

    for _ in range(2):
        packed = torch.full_like(ref_packed, -1)
        idx = torch.full_like(ref_idx, -1)
        rc = _noalloc(lib, qc, kc, qb, qb, topk, packed, idx, stream)
        assert rc == 0, lib.sb_last_error()
        torch.cuda.synchronize(dev)
        assert torch.equal(packed, ref_packed)
        assert torch.equal(idx, ref_idx)


def test_noalloc_route_rejects_rows_larger_than_the_scratch(cuda_device):
    lib = _lib.load()
    # H * candidates = 1024 * 8000 floats exceeds SB_ROUTE_NOALLOC_SCRATCH_FLOATS (4M floats);
    # the size check runs before any pointer is touched.
    dummy = ctypes.c_void_p(256)
    rc = lib.sb_route_topk_noalloc(dummy, dummy, _lib.BF16, 1, 1, 8000, 1024, 128, 8000, 800, 1.0, dummy, None,
                                   None)
    assert rc == -1
    assert "scratch array" in lib.sb_last_error().decode()
