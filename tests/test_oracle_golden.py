"""The CPU oracle pinned against fixtures produced by the reference's own code
(tests/golden/make_golden.py): Top-K route sets, anchor-weighted summaries and the
explicit exact/summary attention."""
import hashlib
import json
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import oracle
from spark_h3_b200.synthetic import make_qkv

GOLDEN = Path(__file__).resolve().parent / "golden"


def digest(t: torch.Tensor) -> str:
    t = t.contiguous()
    raw = t.view(torch.int16).numpy() if t.dtype == torch.bfloat16 else t.numpy()
    return hashlib.sha256(raw.tobytes()).hexdigest()


def host(t: torch.Tensor) -> oracle.Tensor:
    if t.dtype == torch.bfloat16:
        return oracle.Tensor(t.contiguous().view(torch.int16).numpy().view(np.uint16), "bfloat16")
    return oracle.Tensor(t.contiguous().numpy(), "float32")


@pytest.mark.parametrize("name", ["config0", "bf16_d128"])
def test_oracle_route_matches_reference_route(name):
    g = np.load(GOLDEN / f"route_{name}.npz")
    meta = json.loads(str(g["meta"]))
    dtype = torch.float32 if "float32" in meta["dtype"] else torch.bfloat16
    q, k, _ = make_qkv(tuple(meta["grid"]), meta["heads"], meta["dim"], seed=meta["seed"], dtype=dtype,
                       q_scale=meta["q_scale"])
    assert digest(q) == str(g["q_digest"]) and digest(k) == str(g["k_digest"]), "input generator drifted"
    res = oracle.spark_layer(host(q), host(k), host(k), block=64, topk_ratio=0.1, attention=False)
    assert res["topk"] == int(g["target"])
    ref = g["route"].astype(bool)                          # [B, QB, H, C]
    ours = np.zeros_like(ref)
    for idx in np.ndindex(res["indices"].shape[:3]):
        ours[idx][res["indices"][idx]] = True
    differ = (ours != ref).any(-1)
    # Rows may differ only where the k-th and (k+1)-th reference scores are a rounding apart
    # (the two implementations sum the same fp32 products in different orders).
    gap = g["gap"]
    assert np.all(gap[differ] < 1e-5), gap[differ]
    assert differ.mean() < 0.01


def test_oracle_summaries_match_reference_kernel():
    g = np.load(GOLDEN / "summaries.npz")
    gen = torch.Generator().manual_seed(17)
    q = torch.randn(1, 1000, 2, 128, generator=gen) * 128 ** -0.5
    k = torch.randn(1, 1000, 2, 128, generator=gen)
    v = torch.randn(1, 1000, 2, 128, generator=gen)
    assert digest(q) == str(g["q_digest"]) and digest(k) == str(g["k_digest"]) and digest(v) == str(g["v_digest"])
    ak, av, lm = oracle.summaries(g["a"][:, 0], host(k), host(v), 64)
    np.testing.assert_allclose(ak, g["ak"][:, 0], atol=2e-5, rtol=1e-4)
    np.testing.assert_allclose(av, g["av"][:, 0], atol=2e-5, rtol=1e-4)
    np.testing.assert_allclose(lm, g["lm"][:, 0], atol=2e-5, rtol=1e-5)


def test_oracle_attention_matches_reference_formula():
    s = np.load(GOLDEN / "summaries.npz")
    g = np.load(GOLDEN / "attention.npz")
    gen = torch.Generator().manual_seed(17)
    q = torch.randn(1, 1000, 2, 128, generator=gen) * 128 ** -0.5
    k = torch.randn(1, 1000, 2, 128, generator=gen)
    v = torch.randn(1, 1000, 2, 128, generator=gen)
    route = g["route"].astype(bool)                        # [QB_all, H, NB]
    nb = route.shape[-1]
    words = -(-nb // 32)
    packed = np.zeros((1, route.shape[0], 2, words), dtype=np.int64)
    for qb in range(route.shape[0]):
        for h in range(2):
            for kb in np.nonzero(route[qb, h])[0]:
                packed[0, qb, h, kb >> 5] |= 1 << (kb & 31)
    packed = packed.astype(np.uint32).view(np.int32)
    out, _ = oracle.sparse_attention(host(q), host(k), host(v), 64, packed, s["ak"][:, 0], s["av"][:, 0],
                                     s["lm"][:, 0], query_tokens=960, sink_first=15, sink_last=16)
    rows = g["rows"]
    np.testing.assert_allclose(out[0, rows], g["out"], atol=1e-5, rtol=1e-4)


def test_pooled_tail_oracle_with_every_block_exact_is_dense_attention():
    """With Top-K ratio 1 every block is exact, the pooled tails are empty and the layer is
    plain softmax attention (the reference checks the same identity on the GPU,
    tests/test_spark_installer.py:446-485)."""
    import torch

    from spark_h3_b200.synthetic import make_qkv

    q, k, v = make_qkv((2, 8, 16), 1, 128, seed=3, dtype=torch.float32, q_scale=128 ** -0.5)
    t = lambda x: oracle.Tensor(x.numpy(), "float32")
    qf, kf, vf = (x[0, :, 0].double() for x in (q, k, v))
    p = torch.softmax(qf @ kf.T * 128 ** -0.5, dim=-1)
    dense = (p @ vf).numpy()
    for granularity in ("block", "block8x8"):
        ref = oracle.spark_layer(t(q), t(k), t(v), block=64, topk_ratio=1.0, tail_granularity=granularity)
        np.testing.assert_allclose(ref["out"][0, :, 0], dense, atol=1e-5)


def test_oracle_route_matches_reference_route_at_config1():
    """Production size: every (query block, head) row of the oracle's route at BASELINE
    config 1 with 64-token blocks (62,496 rows of 1953 candidates, k = 195) equals the
    reference's own fp32 route, except rows where the reference's k-th and (k+1)-th scores
    are exactly equal."""
    import _config1

    fx = _config1.fixture()
    q, k = _config1.inputs(with_v=False)
    T = q.shape[1]
    candidates, nb = T // 64, -(-T // 64)
    qc = oracle.block_means(_config1.host(q), 64)
    kc = oracle.key_means(_config1.host(k), 64)
    idx, _ = oracle.topk(oracle.scores(qc, kc, candidates, candidates), int(fx["target"]), nb)
    differ = _config1.compare_with_reference(idx, fx)
    assert differ.size == candidates * _config1.HEADS


def test_oracle_head_budgets_match_reference():
    """route_with_head_budgets (head_budget.py:7-19): per-head budgets, including 0 and one
    above the candidate count, with every cut inside a group of equal scores, and on the fp32
    policy scores of synthetic Q/K with a context suffix."""
    g = np.load(GOLDEN / "head_budget.npz")
    scores = g["ties_scores"]
    cand = int(g["ties_candidates"])
    nb = scores.shape[-1]
    idx, packed = oracle.topk_head_budgets(np.ascontiguousarray(scores[..., :cand]), g["ties_budgets"], nb)
    ref = g["ties_route"].astype(bool)
    kb = np.arange(nb)
    ours = ((packed[..., kb >> 5].astype(np.int64) >> (kb & 31)) & 1).astype(bool)
    ours[..., cand:] = True  # the partial video block (video % 64 != 0) stays exact
    np.testing.assert_array_equal(ours, ref)
    budgets = np.clip(g["ties_budgets"], 0, cand)
    assert np.array_equal((idx >= 0).sum(-1)[0, 0], budgets)

    meta = json.loads(str(g["pipe_meta"]))
    q, k, v = make_qkv(tuple(meta["grid"]), meta["heads"], meta["dim"], seed=meta["seed"], dtype=torch.bfloat16,
                       q_scale=meta["q_scale"])
    assert digest(q) == str(g["pipe_q_digest"]) and digest(k) == str(g["pipe_k_digest"])
    video = int(g["pipe_video"])
    res = oracle.spark_layer(host(q), host(k), host(v), block=64, topk_ratio=0.1, video_tokens=video,
                             attention=False, head_budgets=g["pipe_budgets"])
    nb = -(-q.shape[1] // 64)
    kb = np.arange(nb)
    ours = ((res["packed"][..., kb >> 5].astype(np.int64) >> (kb & 31)) & 1).astype(bool)
    ours |= (kb >= res["sink_first"]) & (kb < res["sink_last"])
    # The reference also routes the partial final video query block; with the dense tail its
    # rows attend every key, so the routed query blocks are compared.
    routed = res["packed"].shape[1]
    np.testing.assert_array_equal(ours, g["pipe_route"][:, :routed].astype(bool))
