"""The allocation-free route entry point, sb_route_topk_noalloc, against sb_route_topk.

Callers that cannot hand the library a device workspace (a host binding only this C ABI
through a thin FFI with no device allocator, or a loop that cannot afford the device
synchronisation of cudaMalloc) use the variant whose score scratch is a fixed file-scope
device array.  Both are called here through the C ABI on the same inputs; the route is
integer output, so the comparison is exact, and the variant is called twice in a row to show
that the shared scratch left by one call does not leak into the next.  The cases cover one
and two batch entries, bf16 and fp32 key means, head dims 128 and 64, and a size whose
scores need two passes through the scratch array.

This file is named to be collected last, so a run that stops at the first failure has
already run every other test.
"""
import math

import pytest
import torch

from spark_h3_b200 import _lib, ops
from spark_h3_b200.synthetic import make_qkv

pytestmark = pytest.mark.gpu


def _means(dev, grid, heads, head_dim, dtype, block, batch):
    """Query means [B, NB, H, D] fp32 and key means [B, NB, H, D] in the input dtype."""
    qcs, kcs = [], []
    for b in range(batch):
        q, k, _ = make_qkv(grid, heads, head_dim, seed=9 + b, device=dev, dtype=dtype, q_scale=head_dim ** -0.5)
        qcs.append(ops.pool_queries(q, block))
        kcs.append(ops.pool_keys_summaries(k, None, None, block, want_summaries=False)[0])
    return torch.cat(qcs).contiguous(), torch.cat(kcs).contiguous(), q.shape[1]


@pytest.mark.parametrize("grid,heads,head_dim,dtype,block,batch", [
    ((4, 16, 33), 2, 128, torch.bfloat16, 128, 1),
    # 8 heads x 800 candidate blocks x 800 query blocks = 5.1M scores, more than the
    # 4M-float scratch: the variant works through two chunks.
    ((8, 40, 160), 8, 128, torch.bfloat16, 64, 1),
    # two batch entries: the per-entry offsets of the key and query means
    ((4, 16, 40), 2, 128, torch.bfloat16, 64, 2),
    # fp32 key means at head dim 64 (config 0's shape)
    ((4, 32, 32), 4, 64, torch.float32, 64, 2),
])
def test_noalloc_route_equals_workspace_route(cuda_device, grid, heads, head_dim, dtype, block, batch):
    dev = cuda_device
    qc, kc, T = _means(dev, grid, heads, head_dim, dtype, block, batch)
    qb = T // block
    nb = math.ceil(T / block)
    topk = ops.target_topk(0.1, qb)
    code = _lib.BF16 if dtype == torch.bfloat16 else _lib.F32
    lib = _lib.load()
    stream = torch.cuda.current_stream(dev).cuda_stream

    words = math.ceil(nb / 32)
    ref_packed = torch.empty((batch, qb, heads, words), device=dev, dtype=torch.int32)
    ref_idx = torch.empty((batch, qb, heads, topk), device=dev, dtype=torch.int32)
    workspace = torch.empty(lib.sb_route_workspace_bytes(batch, qb, heads, qb), device=dev, dtype=torch.uint8)
    rc = lib.sb_route_topk(qc.data_ptr(), kc.data_ptr(), code, batch, qb, nb, heads, head_dim, qb, topk,
                           ops.scale_log2(head_dim), workspace.data_ptr(), ref_packed.data_ptr(), ref_idx.data_ptr(),
                           stream)
    assert rc == 0, lib.sb_last_error()

    for _ in range(2):
        packed = torch.full_like(ref_packed, -1)
        idx = torch.full_like(ref_idx, -1)
        rc = lib.sb_route_topk_noalloc(qc.data_ptr(), kc.data_ptr(), code, batch, qb, nb, heads, head_dim, qb, topk,
                                       ops.scale_log2(head_dim), packed.data_ptr(), idx.data_ptr(), stream)
        assert rc == 0, lib.sb_last_error()
        torch.cuda.synchronize(dev)
        assert torch.equal(packed, ref_packed)
        assert torch.equal(idx, ref_idx)


def test_noalloc_route_rejects_rows_larger_than_the_scratch(cuda_device):
    # 513 heads x 8192 candidate blocks = 4.2M scores per query block, more than
    # SB_ROUTE_NOALLOC_SCRATCH_FLOATS (4M floats).  Every buffer is a real device allocation
    # of the declared shape, and the call is refused before any launch.
    dev = cuda_device
    heads, nb, d = 513, 8192, 64
    qc = torch.zeros((1, nb, heads, d), device=dev, dtype=torch.float32)
    kc = torch.zeros((1, nb, heads, d), device=dev, dtype=torch.bfloat16)
    packed = torch.zeros((1, 1, heads, nb // 32), device=dev, dtype=torch.int32)
    lib = _lib.load()
    rc = lib.sb_route_topk_noalloc(qc.data_ptr(), kc.data_ptr(), _lib.BF16, 1, 1, nb, heads, d, nb, 800, 1.0,
                                   packed.data_ptr(), None, torch.cuda.current_stream(dev).cuda_stream)
    assert rc == -1
    message = lib.sb_last_error().decode()
    assert message.startswith("sb_route_topk_noalloc:") and "scratch array" in message
    assert torch.count_nonzero(packed) == 0
