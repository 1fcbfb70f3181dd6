"""GPU parity of every hot-path kernel against the CPU oracle (bit-exact for integer
outputs and block means, within stated tolerances for floating-point outputs)."""
import math

import numpy as np
import pytest
import torch

from oracle import oracle
from spark_h3_b200 import ops
from spark_h3_b200.synthetic import make_qkv

pytestmark = pytest.mark.gpu

# bf16 attention tolerance (north star): max-abs <= 2e-2 and cosine >= 0.9995.
BF16_MAX_ABS = 2e-2
BF16_MIN_COS = 0.9995
F32_MAX_ABS = 1e-4


def to_oracle(t: torch.Tensor) -> oracle.Tensor:
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return oracle.Tensor(t.view(torch.int16).numpy().view(np.uint16), "bfloat16")
    return oracle.Tensor(t.numpy(), "float32")


def as_np(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def cosine(a: np.ndarray, b: np.ndarray) -> float:
    a = a.astype(np.float64).ravel()
    b = b.astype(np.float64).ravel()
    return float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b)))


CASES = [
    # (grid, heads, head_dim, dtype, block, q_scale)
    ((4, 32, 32), 4, 64, torch.float32, 64, 1.0),              # config 0 shape
    ((4, 16, 33), 2, 128, torch.bfloat16, 128, 128 ** -0.5),   # partial 128-block tail
    ((3, 16, 32), 2, 128, torch.bfloat16, 64, 128 ** -0.5),    # 64-token blocks on tensor cores
]


@pytest.mark.parametrize("grid,heads,head_dim,dtype,block,q_scale", CASES)
def test_route_is_bit_exact(cuda_device, grid, heads, head_dim, dtype, block, q_scale):
    q, k, v = make_qkv(grid, heads, head_dim, seed=3, dtype=dtype, q_scale=q_scale)
    oq, ok_, ov = to_oracle(q), to_oracle(k), to_oracle(v)
    ref = oracle.spark_layer(oq, ok_, ov, block=block, topk_ratio=0.1, attention=False)
    out, route = ops.spark_layer(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), block=block,
                                 topk_ratio=0.1, return_route=True)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(as_np(route["qc"]), ref["qc"])
    np.testing.assert_array_equal(as_np(route["kc"]), ref["kc"])
    np.testing.assert_array_equal(as_np(route["anchor"]), ref["anchor"])
    np.testing.assert_array_equal(route["indices"].cpu().numpy(), ref["indices"])
    np.testing.assert_array_equal(route["packed"].cpu().numpy(), ref["packed"])
    assert route["topk"] == ref["topk"]


@pytest.mark.parametrize("grid,heads,head_dim,dtype,block,q_scale", CASES)
def test_summaries_match_oracle(cuda_device, grid, heads, head_dim, dtype, block, q_scale):
    q, k, v = make_qkv(grid, heads, head_dim, seed=5, dtype=dtype, q_scale=q_scale)
    anchor = ops.query_anchor(ops.pool_queries(q.to(cuda_device), block), block,
                              q.shape[1] // block, dtype)
    _, ak, av, lm = ops.pool_keys_summaries(k.to(cuda_device), v.to(cuda_device), anchor, block)
    ref_ak, ref_av, ref_lm = oracle.summaries(as_np(anchor), to_oracle(k), to_oracle(v), block)
    tol = 1.6e-2 if dtype == torch.bfloat16 else 1e-5
    np.testing.assert_allclose(as_np(ak), ref_ak, atol=tol, rtol=tol)
    np.testing.assert_allclose(as_np(av), ref_av, atol=tol, rtol=tol)
    np.testing.assert_allclose(as_np(lm), ref_lm, atol=2e-3 if dtype == torch.bfloat16 else 1e-5, rtol=1e-3)


def _attention_case(cuda_device, grid, heads, head_dim, dtype, block, q_scale, *, video=None, local_radius=-1,
                    seed=7):
    q, k, v = make_qkv(grid, heads, head_dim, seed=seed, dtype=dtype, q_scale=q_scale)
    T = q.shape[1]
    video = T if video is None else video
    ref = oracle.spark_layer(to_oracle(q), to_oracle(k), to_oracle(v), block=block, topk_ratio=0.1,
                             video_tokens=video, local_radius=local_radius)
    dev = cuda_device
    packed = torch.from_numpy(ref["packed"]).to(dev)
    cast = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev, dtype)
    ak, av = cast(ref["ak"]), cast(ref["av"])
    lm = torch.from_numpy(ref["lm"]).to(dev)
    out, lse = ops.sparse_attention(q.to(dev), k.to(dev), v.to(dev), block, packed, ak, av, lm,
                                    query_tokens=ref["query_tokens"], sink_first=ref["sink_first"],
                                    sink_last=ref["sink_last"], local_radius=local_radius, want_lse=True)
    torch.cuda.synchronize()
    assert ops.read_device_status(dev) == 0
    return as_np(out), as_np(lse), ref["out"], ref["lse"]


def _check(out, ref, dtype):
    assert np.isfinite(out).all()
    err = np.abs(out - ref).max()
    if dtype == torch.bfloat16:
        assert err <= BF16_MAX_ABS, err
        assert cosine(out, ref) >= BF16_MIN_COS
    else:
        assert err <= F32_MAX_ABS, err


@pytest.mark.parametrize("grid,heads,head_dim,dtype,block,q_scale", CASES)
def test_sparse_attention_matches_oracle(cuda_device, grid, heads, head_dim, dtype, block, q_scale):
    out, lse, ref, ref_lse = _attention_case(cuda_device, grid, heads, head_dim, dtype, block, q_scale)
    _check(out, ref, dtype)
    np.testing.assert_allclose(lse, ref_lse, atol=2e-3 if dtype == torch.bfloat16 else 1e-5, rtol=1e-4)


@pytest.mark.parametrize("block", [64, 128])
def test_sparse_attention_context_sink_and_dense_suffix(cuda_device, block):
    # 2112 video tokens followed by 150 context tokens: the context blocks are forced
    # exact, and every row past the last complete video block is attended densely.
    grid = (4, 16, 33)
    q, k, v = make_qkv(grid, 2, 128, seed=11, dtype=torch.bfloat16, q_scale=128 ** -0.5)
    extra = make_qkv((1, 10, 15), 2, 128, seed=12, dtype=torch.bfloat16, q_scale=128 ** -0.5)
    q, k, v = (torch.cat((a, b), dim=1) for a, b in zip((q, k, v), extra))
    T = q.shape[1]
    video = 2112
    ref = oracle.spark_layer(to_oracle(q), to_oracle(k), to_oracle(v), block=block, topk_ratio=0.1,
                             video_tokens=video)
    out = ops.spark_layer(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), block=block, topk_ratio=0.1,
                          video_tokens=video)
    torch.cuda.synchronize()
    assert ref["sink_last"] > ref["sink_first"]
    _check(as_np(out), ref["out"], torch.bfloat16)


def test_sparse_attention_local_radius(cuda_device):
    out, _, ref, _ = _attention_case(cuda_device, (3, 16, 32), 2, 128, torch.bfloat16, 64, 128 ** -0.5,
                                     local_radius=1)
    _check(out, ref, torch.bfloat16)


def test_tensor_core_kernel_agrees_with_simt_kernel(cuda_device):
    # The same bf16 problem through the sm100 kernel (D = 128) and through the SIMT kernel
    # (fed float32 copies): both are GPU paths of the library and must agree.
    q, k, v = make_qkv((2, 16, 40), 2, 128, seed=21, dtype=torch.bfloat16, q_scale=128 ** -0.5)
    dev = cuda_device
    out_tc, route = ops.spark_layer(q.to(dev), k.to(dev), v.to(dev), block=128, return_route=True)
    f = lambda t: t.to(dev).float()
    out_simt, _ = ops.sparse_attention(f(q), f(k), f(v), 128, route["packed"], route["ak"].float(),
                                       route["av"].float(), route["lm"], query_tokens=route["query_tokens"],
                                       sink_first=route["sink_first"], sink_last=route["sink_last"])
    torch.cuda.synchronize()
    _check(as_np(out_tc), as_np(out_simt), torch.bfloat16)


def test_headwise_permute_roundtrip(cuda_device):
    gen = torch.Generator().manual_seed(4)
    B, T, H, D, video = 1, 1000, 3, 128, 900
    x = torch.randn(B, T, H, D, generator=gen).to(torch.bfloat16)
    perm = torch.stack([torch.randperm(video, generator=gen) for _ in range(H)])[None]
    inv = torch.argsort(perm, dim=-1)
    dev = cuda_device
    y = ops.headwise_permute(x.to(dev), perm.to(dev), video)
    z = ops.headwise_permute(y, inv.to(dev), video)
    expected = x.clone()
    for h in range(H):
        expected[0, :video, h] = x[0, perm[0, h], h]
    assert torch.equal(y.cpu(), expected)
    assert torch.equal(z.cpu(), x)
    y32 = ops.headwise_permute(x.to(dev), perm.to(dev).to(torch.int32), video)
    assert torch.equal(y32.cpu(), expected)


@pytest.mark.parametrize("block", [64, 128])
def test_pad_tail_mode_matches_oracle(cuda_device, block):
    # 2100 video tokens (a partial final block) followed by 162 context tokens; tail mode
    # "pad" routes the final video block padded with its own mean and attends the context
    # rows that padded it densely.
    q, k, v = make_qkv((4, 16, 33), 2, 128, seed=31, dtype=torch.bfloat16, q_scale=128 ** -0.5)
    extra = make_qkv((1, 10, 15), 2, 128, seed=32, dtype=torch.bfloat16, q_scale=128 ** -0.5)
    q, k, v = (torch.cat((a, b), dim=1) for a, b in zip((q, k, v), extra))
    video = 2100
    ref = oracle.spark_layer(to_oracle(q), to_oracle(k), to_oracle(v), block=block, topk_ratio=0.1,
                             video_tokens=video, tail_mode="pad")
    out, route = ops.spark_layer(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), block=block,
                                 topk_ratio=0.1, video_tokens=video, tail_mode="pad", return_route=True)
    torch.cuda.synchronize()
    assert route["query_tokens"] == ref["query_tokens"] == -(-video // block) * block
    np.testing.assert_array_equal(as_np(route["qc"]), ref["qc"])
    np.testing.assert_array_equal(route["indices"].cpu().numpy(), ref["indices"])
    _check(as_np(out), ref["out"], torch.bfloat16)
    # The dense rows differ from what the sparse prefix alone would give them.
    dense = ops.spark_layer(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), block=block,
                            topk_ratio=0.1, video_tokens=video)
    torch.cuda.synchronize()
    assert not torch.equal(dense[:, :video].cpu(), out[:, :video].cpu())
    _check(as_np(out)[:, video:], as_np(dense)[:, video:], torch.bfloat16)


@pytest.mark.parametrize("block", [64, 128])
def test_legacy_full_query_matches_oracle(cuda_device, block):
    # sol_legacy_full_query (spark_integration.py:925-933): the partial final video block is
    # routed with the mean of all its rows (video and context), evaluated sparsely, and its
    # context rows are then attended densely with every row after them.
    q, k, v = make_qkv((4, 16, 33), 2, 128, seed=31, dtype=torch.bfloat16, q_scale=128 ** -0.5)
    extra = make_qkv((1, 10, 15), 2, 128, seed=32, dtype=torch.bfloat16, q_scale=128 ** -0.5)
    q, k, v = (torch.cat((a, b), dim=1) for a, b in zip((q, k, v), extra))
    video = 2100
    ref = oracle.spark_layer(to_oracle(q), to_oracle(k), to_oracle(v), block=block, topk_ratio=0.1,
                             video_tokens=video, tail_mode="legacy_full")
    out, route = ops.spark_layer(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), block=block,
                                 topk_ratio=0.1, video_tokens=video, tail_mode="legacy_full", return_route=True)
    torch.cuda.synchronize()
    assert route["query_tokens"] == ref["query_tokens"] == -(-video // block) * block
    np.testing.assert_array_equal(as_np(route["qc"]), ref["qc"])
    np.testing.assert_array_equal(route["indices"].cpu().numpy(), ref["indices"])
    _check(as_np(out), ref["out"], torch.bfloat16)
    # Through the attention seam with the reference's config flag.
    from spark_h3_b200.attention import spark_attention_bthd
    from spark_h3_b200.config import H3SparseAttentionConfig
    from spark_h3_b200.layout import PackedLayout
    from spark_h3_b200.processor import _Controller

    T = q.shape[1]
    cfg = H3SparseAttentionConfig.spark(num_inference_steps=4, mode="reweight_only", sol_route_topk_ratio=0.1,
                                        sol_legacy_full_query=True, sol_block_size=block)
    ids = torch.arange(T)
    layout = PackedLayout(permutation=ids, inverse_permutation=ids, grid=(1, 1, video), video_tokens=video,
                          sequence_length=T, video_positions=torch.zeros(video, 3, dtype=torch.long))
    seam = spark_attention_bthd(_Controller(cfg), q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), layout, 0)
    torch.cuda.synchronize()
    assert torch.equal(seam.cpu(), out.cpu())


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_dense_rows_attention_window(cuda_device, dtype):
    q, k, v = make_qkv((3, 16, 32), 2, 128, seed=41, dtype=dtype, q_scale=128 ** -0.5)
    dev = cuda_device
    T = q.shape[1]
    out = torch.full_like(q, 7.0).to(dev)
    lse = torch.full((1, T, 2), 7.0, device=dev)
    ops.dense_rows_attention(q.to(dev), k.to(dev), v.to(dev), 70, 333, out, lse=lse)
    torch.cuda.synchronize()
    ref, ref_lse = oracle.sparse_attention(to_oracle(q), to_oracle(k), to_oracle(v), 64, np.zeros((1, 0, 2, 1)),
                                           np.zeros((1, 2, 24, 128)), np.zeros((1, 2, 24, 128)),
                                           np.zeros((1, 2, 24)), 0, 0, 0, rows=slice(70, 333))
    o = as_np(out)
    assert (o[:, :70] == 7.0).all() and (o[:, 333:] == 7.0).all()
    _check(o[:, 70:333], ref[:, 70:333], dtype)
    np.testing.assert_allclose(as_np(lse)[:, 70:333], ref_lse[:, 70:333], atol=2e-3, rtol=1e-4)
    assert (as_np(lse)[:, :70] == 7.0).all() and (as_np(lse)[:, 333:] == 7.0).all()


@pytest.mark.parametrize("summary_math,logmass_key", [("tensorcore", "pre_round"), ("comfy_fp32", "stored"),
                                                      ("comfy_fp32", "pre_round")])
def test_summary_ablations_match_oracle(cuda_device, summary_math, logmass_key):
    """The reference's summary numerics ablations (processor.py:61-68): the oracle restated
    with the same switch, and each switch changes what it should (bit-for-bit comparison
    with the default summaries on the GPU)."""
    grid, heads, block = (3, 16, 32), 2, 64
    q, k, v = make_qkv(grid, heads, 128, seed=5, dtype=torch.bfloat16, q_scale=128 ** -0.5)
    dev = cuda_device
    anchor = ops.query_anchor(ops.pool_queries(q.to(dev), block), block, q.shape[1] // block, torch.float32)
    _, ak, av, lm = ops.pool_keys_summaries(k.to(dev), v.to(dev), anchor, block, summary_math=summary_math,
                                            logmass_key=logmass_key)
    _, ak0, av0, lm0 = ops.pool_keys_summaries(k.to(dev), v.to(dev), anchor, block)
    ref_ak, ref_av, ref_lm = oracle.summaries(as_np(anchor), to_oracle(k), to_oracle(v), block,
                                              summary_math=summary_math, logmass_key=logmass_key)
    np.testing.assert_allclose(as_np(ak), ref_ak, atol=1.6e-2, rtol=1.6e-2)
    np.testing.assert_allclose(as_np(av), ref_av, atol=1.6e-2, rtol=1.6e-2)
    np.testing.assert_allclose(as_np(lm), ref_lm, atol=2e-3, rtol=1e-3)
    if summary_math == "comfy_fp32":
        assert not torch.equal(ak, ak0) and not torch.equal(av, av0)
    else:
        assert torch.equal(ak, ak0) and torch.equal(av, av0)
    assert not torch.equal(lm, lm0)


def test_exact_only_attention_matches_oracle(cuda_device):
    """Without summaries the kernel attends the exact blocks only (the first stage of the
    block tails), for both the tensor-core and the SIMT kernel."""
    q, k, v = make_qkv((3, 16, 32), 2, 128, seed=51, dtype=torch.bfloat16, q_scale=128 ** -0.5)
    ref = oracle.spark_layer(to_oracle(q), to_oracle(k), to_oracle(v), block=64, topk_ratio=0.1, attention=False)
    dev = cuda_device
    packed = torch.from_numpy(ref["packed"]).to(dev)
    exp_out, exp_lse = oracle.sparse_attention(to_oracle(q), to_oracle(k), to_oracle(v), 64, ref["packed"], None,
                                               None, None, ref["query_tokens"], ref["sink_first"], ref["sink_last"])
    for cast in (lambda t: t.to(dev), lambda t: t.to(dev).float()):
        out, lse = ops.sparse_attention(cast(q), cast(k), cast(v), 64, packed, None, None, None,
                                        query_tokens=ref["query_tokens"], sink_first=ref["sink_first"],
                                        sink_last=ref["sink_last"], want_lse=True)
        torch.cuda.synchronize()
        _check(as_np(out), exp_out, torch.bfloat16)
        np.testing.assert_allclose(as_np(lse), exp_lse, atol=2e-3, rtol=1e-4)


@pytest.mark.parametrize("granularity", ["block", "block8x8"])
@pytest.mark.parametrize("block", [64, 128])
def test_pooled_tails_match_oracle(cuda_device, granularity, block):
    """Tail granularities "block" and "block8x8" (sol_numerator_virtual_q.py:415-499) with
    context sinks and a dense suffix: route bit-exact, output within the bf16 tolerance."""
    q, k, v = make_qkv((4, 16, 33), 2, 128, seed=61, dtype=torch.bfloat16, q_scale=128 ** -0.5)
    extra = make_qkv((1, 10, 15), 2, 128, seed=62, dtype=torch.bfloat16, q_scale=128 ** -0.5)
    q, k, v = (torch.cat((a, b), dim=1) for a, b in zip((q, k, v), extra))
    video = 2112
    ref = oracle.spark_layer(to_oracle(q), to_oracle(k), to_oracle(v), block=block, topk_ratio=0.1,
                             video_tokens=video, tail_granularity=granularity)
    out, route = ops.spark_layer(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), block=block,
                                 topk_ratio=0.1, video_tokens=video, tail_granularity=granularity, return_route=True)
    torch.cuda.synchronize()
    assert ops.read_device_status(cuda_device) == 0
    np.testing.assert_array_equal(route["indices"].cpu().numpy(), ref["indices"])
    _check(as_np(out), ref["out"], torch.bfloat16)
    # The pooled tail differs from the per-row summaries of the default granularity.
    per_row = ops.spark_layer(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), block=block, topk_ratio=0.1,
                              video_tokens=video)
    torch.cuda.synchronize()
    assert not torch.equal(per_row.cpu(), out.cpu())


@pytest.mark.parametrize("block,granularity", [(64, "query"), (128, "query"), (64, "block")])
def test_batch_of_two_matches_oracle(cuda_device, block, granularity):
    """Two batch entries with different content through one call: routes bit-exact and
    outputs within tolerance per entry (every kernel indexes the batch explicitly)."""
    parts = [make_qkv((3, 16, 33), 2, 128, seed=s, dtype=torch.bfloat16, q_scale=128 ** -0.5) for s in (71, 72)]
    q, k, v = (torch.cat([p[i] for p in parts], dim=0) for i in range(3))
    ref = oracle.spark_layer(to_oracle(q), to_oracle(k), to_oracle(v), block=block, topk_ratio=0.1,
                             tail_granularity=granularity)
    out, route = ops.spark_layer(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), block=block,
                                 topk_ratio=0.1, tail_granularity=granularity, return_route=True)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(route["indices"].cpu().numpy(), ref["indices"])
    assert not np.array_equal(ref["indices"][0], ref["indices"][1])
    for b in range(2):
        _check(as_np(out)[b], ref["out"][b], torch.bfloat16)


def _long_sequence_case(T: int, block: int, seed: int):
    """Seeded bf16 Q/K/V for one head, a random route (eight routed key blocks per query
    block), and random summaries: sized so that the route tables crowd the shared memory."""
    g = torch.Generator().manual_seed(seed)
    q, k, v = (torch.randn((1, T, 1, 128), generator=g).to(torch.bfloat16) for _ in range(3))
    q = (q.float() * 128 ** -0.5).to(torch.bfloat16)
    nb = -(-T // block)
    words = -(-nb // 32)
    rng = np.random.default_rng(seed)
    bits = np.zeros((1, nb, 1, words * 32), dtype=np.uint8)
    for qb in range(nb):
        bits[0, qb, 0, rng.choice(nb, 8, replace=False)] = 1
        bits[0, qb, 0, qb] = 1
    packed = np.packbits(bits, axis=-1, bitorder="little").view(np.int32)
    ak = (rng.standard_normal((1, 1, nb, 128)) * 0.5).astype(np.float32)
    av = rng.standard_normal((1, 1, nb, 128)).astype(np.float32)
    lm = rng.uniform(0.0, 4.0, (1, 1, nb)).astype(np.float32)
    return q, k, v, packed, ak, av, lm


def test_long_sequence_two_stage_value_ring(cuda_device):
    # 400,037 tokens in 64-token blocks: the per-sequence tables leave room for two V stages
    # only.  Rows of the first, a middle and the ragged last query tile are checked; the last
    # tile holds routed rows and the 37 dense-suffix rows past the last whole block.
    T, block = 400_037, 64
    routed = T // block * block
    q, k, v, packed, ak, av, lm = _long_sequence_case(T, block, seed=31)
    dev = cuda_device
    bf = lambda a: torch.from_numpy(a).to(dev, torch.bfloat16)
    ak_d, av_d = bf(ak), bf(av)
    out, lse = ops.sparse_attention(q.to(dev), k.to(dev), v.to(dev), block, torch.from_numpy(packed).to(dev),
                                    ak_d, av_d, torch.from_numpy(lm).to(dev), query_tokens=routed,
                                    sink_first=0, sink_last=0, want_lse=True)
    torch.cuda.synchronize()
    assert ops.read_device_status(dev) == 0
    out, lse = as_np(out), as_np(lse)
    ak_r, av_r = as_np(ak_d), as_np(av_d)  # the summaries as the kernel saw them (bf16)
    last = (T - 1) // 128 * 128
    oq, ok_, ov = to_oracle(q), to_oracle(k), to_oracle(v)
    for r0, r1 in ((0, 128), (200_064, 200_192), (last, T)):
        ref, ref_lse = oracle.sparse_attention(oq, ok_, ov, block, packed, ak_r, av_r, lm, routed, 0, 0,
                                               rows=slice(r0, r1))
        _check(out[:, r0:r1], ref[:, r0:r1], torch.bfloat16)
        np.testing.assert_allclose(lse[:, r0:r1], ref_lse[:, r0:r1], atol=2e-3, rtol=1e-4)


def test_sequence_past_shared_memory_limit_fails_loudly(cuda_device):
    # 700,000 tokens in 64-token blocks: even two K stages no longer fit beside the tables;
    # the launcher refuses before any launch and the context stays usable.
    T, block = 700_000, 64
    dev = cuda_device
    nb = -(-T // block)
    q = torch.zeros((1, T, 1, 128), device=dev, dtype=torch.bfloat16)
    packed = torch.zeros((1, nb, 1, -(-nb // 32)), device=dev, dtype=torch.int32)
    ak = torch.zeros((1, 1, nb, 128), device=dev, dtype=torch.bfloat16)
    lm = torch.zeros((1, 1, nb), device=dev, dtype=torch.float32)
    with pytest.raises(RuntimeError, match="too long for the tensor-core kernel"):
        ops.sparse_attention(q, q, q, block, packed, ak, ak, lm, query_tokens=T // block * block, sink_first=0,
                             sink_last=0)
    torch.cuda.synchronize()
    assert ops.read_device_status(dev) == 0


@pytest.mark.parametrize("block", [64, 128])
def test_route_ties_take_the_lowest_block_ids(cuda_device, block):
    # Key blocks repeat with period 4, so every query block sees each distinct score on
    # 1/4 of the candidates: the Top-K cut falls inside a group of exactly equal scores and
    # the lowest block ids of that group are taken (the oracle's stable descending order).
    grid = (4, 16, 32)
    q, k, v = make_qkv(grid, 2, 128, seed=51, dtype=torch.bfloat16, q_scale=128 ** -0.5)
    T = q.shape[1]
    nb = T // block
    k = k.view(1, nb, block, 2, 128)[:, [b % 4 for b in range(nb)]].reshape(1, T, 2, 128).contiguous()
    ref = oracle.spark_layer(to_oracle(q), to_oracle(k), to_oracle(v), block=block, topk_ratio=0.1)
    out, route = ops.spark_layer(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), block=block,
                                 topk_ratio=0.1, return_route=True)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(route["indices"].cpu().numpy(), ref["indices"])
    np.testing.assert_array_equal(route["packed"].cpu().numpy(), ref["packed"])
    # The selection restated from the scores: every block above the k-th score, then the
    # lowest ids among the blocks equal to it.
    topk = ref["topk"]
    sc = ref["scores"].reshape(-1, ref["scores"].shape[-1])
    got = route["indices"].cpu().numpy().reshape(sc.shape[0], topk)
    kth = -np.sort(-sc, axis=-1)[:, topk - 1]
    cut_in_ties = 0
    for row in range(sc.shape[0]):
        above = np.flatnonzero(sc[row] > kth[row])
        tied = np.flatnonzero(sc[row] == kth[row])
        cut_in_ties += len(above) + len(tied) > topk
        expected = np.concatenate([above, tied[:topk - len(above)]])
        np.testing.assert_array_equal(np.sort(got[row]), np.sort(expected))
    assert cut_in_ties == sc.shape[0]  # every row's cut falls inside a group of equal scores
    _check(as_np(out), ref["out"], torch.bfloat16)


def test_all_zero_inputs_match_oracle(cuda_device):
    # Every score, summary logit and attention logit ties: uniform routing by block id,
    # uniform summary weights, and a zero output.
    q = torch.zeros((1, 2048, 2, 128), dtype=torch.bfloat16)
    ref = oracle.spark_layer(to_oracle(q), to_oracle(q), to_oracle(q), block=64, topk_ratio=0.1)
    d = q.to(cuda_device)
    out, route = ops.spark_layer(d, d, d, block=64, topk_ratio=0.1, return_route=True)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(route["indices"].cpu().numpy(), ref["indices"])
    np.testing.assert_array_equal(route["packed"].cpu().numpy(), ref["packed"])
    assert np.all(as_np(out) == 0.0)
    np.testing.assert_array_equal(ref["out"], 0.0)
    assert ops.read_device_status(cuda_device) == 0


@pytest.mark.parametrize("block", [64, 128])
@pytest.mark.parametrize("ties", [False, True])
def test_head_budget_route_matches_oracle(cuda_device, block, ties):
    """Per-head Top-K budgets (head_budget.py:7-19): budgets of 0, inside and above the
    candidate count, a context suffix that keeps every block past the candidates exact, and
    (ties=True) key blocks repeating with period 4 so every cut falls inside equal scores."""
    grid = (2, 16, 40)
    q, k, v = make_qkv(grid, 4, 128, seed=29, dtype=torch.bfloat16, q_scale=128 ** -0.5)
    T = q.shape[1]
    video = T - 100
    if ties:
        nb = T // block
        k = k.view(1, nb, block, 4, 128)[:, [b % 4 for b in range(nb)]].reshape(1, T, 4, 128).contiguous()
    candidates = video // block
    budgets = np.array([3, 0, candidates - 1, candidates + 3], dtype=np.int32)
    ref = oracle.spark_layer(to_oracle(q), to_oracle(k), to_oracle(v), block=block, topk_ratio=0.1,
                             video_tokens=video, head_budgets=budgets)
    out, route = ops.spark_layer(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), block=block,
                                 topk_ratio=0.1, video_tokens=video, return_route=True,
                                 head_budgets=torch.from_numpy(budgets).to(cuda_device))
    torch.cuda.synchronize()
    assert (route["sink_first"], route["sink_last"]) == (ref["sink_first"], ref["sink_last"]) == \
        (candidates, math.ceil(T / block))
    np.testing.assert_array_equal(route["packed"].cpu().numpy(), ref["packed"])
    np.testing.assert_array_equal(route["indices"].cpu().numpy(), ref["indices"])
    counts = (route["indices"].cpu().numpy() >= 0).sum(-1)[0]
    assert np.array_equal(counts, np.broadcast_to(np.minimum(np.clip(budgets, 0, candidates), ref["topk"]),
                                                  counts.shape))
    _check(as_np(out), ref["out"], torch.bfloat16)
