"""This library's outputs against the reference's own GPU kernels on a B200, called from the
installed copy under baseline/_ref (the reference arm's install); skipped where that copy or
its CuTe DSL is absent.
- Attention against SparkReweightForwardSm100 (h3_sparse_attention/spark_reweight_sm100.py,
  reached through sol_numerator_virtual_q.py's virtual_q_attention with
  H3_SPARK_REWEIGHT_FUSED=1) on the same Q/K/V, route, anchors and summaries: the north_star's
  bf16 attention bar, max-abs <= 2e-2 and cosine >= 0.9995.
- Anchors and summaries against build_virtual_anchors and the Triton virtual_summaries
  (sol_numerator_virtual_q.py:93-135, 268-353)."""
from __future__ import annotations

import os
from pathlib import Path

import pytest
import torch

from spark_h3_b200 import ops
from spark_h3_b200.synthetic import make_qkv

pytestmark = pytest.mark.gpu
REF = Path(__file__).resolve().parents[1] / "baseline" / "_ref" / "h3_sparse_attention"


@pytest.fixture(scope="module")
def reference_sm100():
    if not REF.is_dir():
        pytest.skip("the reference is not installed under baseline/_ref")
    try:
        import cutlass.cute as cute
    except ImportError:
        pytest.skip("the CuTe DSL is not importable")
    import sys

    import bench

    compile_, fused, path = cute.compile, os.environ.get("H3_SPARK_REWEIGHT_FUSED"), list(sys.path)
    try:
        yield bench._import_reference_sm100()
    finally:
        cute.compile = compile_
        sys.path[:] = path
        if fused is None:
            os.environ.pop("H3_SPARK_REWEIGHT_FUSED", None)
        else:
            os.environ["H3_SPARK_REWEIGHT_FUSED"] = fused


@pytest.mark.parametrize("grid,heads,topk_ratio", [((4, 16, 33), 4, 0.1), ((2, 32, 64), 2, 0.25)])
def test_attention_matches_the_references_sm100_kernel(cuda_device, reference_sm100, grid, heads, topk_ratio):
    rw, reduce_kv = reference_sm100
    q, k, v = make_qkv(grid, heads, 128, seed=0, device=cuda_device, dtype=torch.bfloat16, q_scale=128 ** -0.5)
    T = q.shape[1]
    n = T // 64
    qc = ops.pool_queries(q, 64)
    anchor = ops.query_anchor(qc, 64, n, q.dtype)
    kc, ak, av, lm = ops.pool_keys_summaries(k, v, anchor, 64)
    topk = ops.target_topk(topk_ratio, n)
    packed, _ = ops.route_topk(qc, kc, n, n, topk)
    ours = ops.sparse_attention(q, k, v, 64, packed, ak, av, lm, query_tokens=T, sink_first=n, sink_last=n,
                                out=torch.empty_like(q))[0]
    ranges = torch.tensor([[0, T]], device=cuda_device, dtype=torch.int64)
    mapping = torch.zeros(n, device=cuda_device, dtype=torch.int64)
    kc_ref, _ = reduce_kv(k, v)
    anchors = rw.build_virtual_anchors(q, ranges)
    ref = rw.virtual_q_attention(q, k, v, virtual_ranges=ranges, leaf_to_virtual=mapping, key_centroids=kc_ref,
                                 route=rw.unpack_packed_route(packed, n), sink_tokens=0, force_local_blocks=False,
                                 virtual_anchors=anchors, precomputed_summaries=rw.virtual_summaries(anchors, k, v))
    torch.cuda.synchronize()
    assert rw.virtual_q_backend(q) == "sm100_fused_virtual_query"
    a, b = ours.float().flatten(), ref.float().flatten()
    assert torch.isfinite(b).all()
    assert float((a - b).abs().max()) <= 2e-2
    assert float((a @ b) / (a.norm() * b.norm())) >= 0.9995


def test_anchor_and_summaries_match_the_references_triton_kernels(cuda_device, reference_sm100):
    """Anchors bit for bit; AK and AV within one bf16 ulp (all but a few elements equal: the
    weighted sums' fp32 order differs); LM within 1e-5.  Config-1 shape with 4 heads."""
    rw, _ = reference_sm100
    q, k, v = make_qkv((31, 48, 84), 4, 128, seed=0, device=cuda_device, dtype=torch.bfloat16, q_scale=128 ** -0.5)
    B, T, H, D = q.shape
    n = T // 64
    anchor = ops.query_anchor(ops.pool_queries(q, 64), 64, n, q.dtype)
    _, ak, av, lm = ops.pool_keys_summaries(k, v, anchor, 64)
    ranges = torch.tensor([[0, T]], device=cuda_device, dtype=torch.int64)
    ref_anchor = rw.build_virtual_anchors(q, ranges)
    rak, rav, rlm = rw.virtual_summaries(ref_anchor, k, v)
    torch.cuda.synchronize()
    assert torch.equal(ref_anchor.reshape(-1), anchor.reshape(-1))
    for ours, ref in ((ak, rak.reshape(ak.shape)), (av, rav.reshape(av.shape))):
        diff = (ours.float() - ref.float()).abs()
        bound = 2.0 ** -7 * torch.maximum(ours.float().abs(), ref.float().abs()) + 1e-6
        assert bool((diff <= bound).all()), float(diff.max())
        assert float((diff == 0).float().mean()) >= 0.9999
    assert float((lm - rlm.reshape(lm.shape)).abs().max()) <= 1e-5
