"""Query-block pairing (sb_route_pair_blocks) and the attention kernel's paired tiles.

With 64-token blocks the tensor-core kernel's 128-row tiles hold two query blocks and do the
exact key work of the union of their route sets; pairing blocks by route overlap shrinks that
union.  The pairs are integers and must equal the oracle's restatement exactly; the attention
with pairs must match the oracle within the bf16 tolerance, and the unpaired kernel within it.
"""
import numpy as np
import pytest
import torch

from oracle import oracle
from spark_h3_b200 import ops
from spark_h3_b200.synthetic import make_qkv

pytestmark = pytest.mark.gpu

BF16_MAX_ABS = 2e-2
BF16_MIN_COS = 0.9995


def _random_route(B, QB, H, nb, per_row, seed, similar=True):
    """Packed routes [B, QB, H, ceil(nb/32)] with `per_row` blocks each; `similar` makes
    nearby query blocks share most of their sets (as a reblocked route does)."""
    rng = np.random.default_rng(seed)
    words = -(-nb // 32)
    bits = np.zeros((B, QB, H, words * 32), np.uint8)
    for b in range(B):
        for h in range(H):
            base = rng.choice(nb, per_row, replace=False)
            for a in range(QB):
                if similar and rng.random() < 0.7:
                    swap = rng.choice(per_row, per_row // 4, replace=False)
                    base = base.copy()
                    base[swap] = rng.choice(nb, len(swap), replace=False)
                    base = np.unique(base)
                    while len(base) < per_row:
                        base = np.unique(np.append(base, rng.integers(nb)))
                else:
                    base = rng.choice(nb, per_row, replace=False)
                bits[b, a, h, base] = 1
    return np.packbits(bits, axis=-1, bitorder="little").view(np.int32)


@pytest.mark.parametrize("B,QB,H,nb,per_row,blocks", [
    (1, 150, 2, 150, 15, 150),    # even count, window reaches past the end
    (2, 201, 3, 300, 30, 199),    # odd count of paired blocks, a longer route than the pairs
    (1, 400, 1, 400, 40, 400),    # several windows
])
def test_pairs_match_oracle(cuda_device, B, QB, H, nb, per_row, blocks):
    packed = _random_route(B, QB, H, nb, per_row, seed=QB + H)
    got = ops.route_pairs(torch.from_numpy(packed).to(cuda_device), blocks).cpu().numpy()
    ref = oracle.block_pairs(packed, blocks)
    assert np.array_equal(got, ref)
    flat = np.sort(got.reshape(B, H, -1), axis=-1)
    expect = np.arange(blocks)
    for b in range(B):
        for h in range(H):
            row = flat[b, h]
            assert np.array_equal(row[row >= 0], expect)  # every block in exactly one tile


def _layer_case(grid, heads, block, seed, video=None, extra=None):
    q, k, v = make_qkv(grid, heads, 128, seed=seed, dtype=torch.bfloat16, q_scale=128 ** -0.5)
    if extra is not None:
        e = make_qkv(extra, heads, 128, seed=seed + 1, dtype=torch.bfloat16, q_scale=128 ** -0.5)
        q, k, v = (torch.cat((a, b2), dim=1) for a, b2 in zip((q, k, v), e))
    return q, k, v


def _check(out, ref):
    out = out.astype(np.float64)
    ref = ref.astype(np.float64)
    assert np.isfinite(out).all()
    assert np.abs(out - ref).max() <= BF16_MAX_ABS
    assert float(out.ravel() @ ref.ravel() / (np.linalg.norm(out) * np.linalg.norm(ref))) >= BF16_MIN_COS


@pytest.mark.parametrize("grid,extra,video", [
    ((3, 16, 32), None, None),             # 24 routed blocks, no suffix
    ((4, 16, 33), (1, 10, 15), 2112),      # 33 routed blocks (odd) and a 150-row dense suffix
])
def test_paired_attention_matches_oracle(cuda_device, grid, extra, video):
    q, k, v = _layer_case(grid, 2, 64, seed=41, extra=extra)
    ref = oracle.spark_layer(oracle.Tensor(q.view(torch.int16).numpy().view(np.uint16), "bfloat16"),
                             oracle.Tensor(k.view(torch.int16).numpy().view(np.uint16), "bfloat16"),
                             oracle.Tensor(v.view(torch.int16).numpy().view(np.uint16), "bfloat16"),
                             block=64, topk_ratio=0.1, video_tokens=video)
    dev = cuda_device
    packed = torch.from_numpy(ref["packed"]).to(dev)
    bf = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev, torch.bfloat16)
    args = (q.to(dev), k.to(dev), v.to(dev), 64, packed, bf(ref["ak"]), bf(ref["av"]), torch.from_numpy(ref["lm"]).to(dev))
    kw = dict(query_tokens=ref["query_tokens"], sink_first=ref["sink_first"], sink_last=ref["sink_last"])
    routed = ref["query_tokens"] // 64
    pairs = ops.route_pairs(packed, routed)
    adjacent = np.arange(2 * pairs.shape[2]).reshape(-1, 2)
    assert not np.array_equal(pairs[0, 0].cpu().numpy(), adjacent)  # the pairing is not the trivial one
    paired, lse_p = ops.sparse_attention(*args, **kw, pairs=pairs, want_lse=True)
    plain, lse_u = ops.sparse_attention(*args, **kw, pair_blocks=False, want_lse=True)
    torch.cuda.synchronize()
    assert ops.read_device_status(dev) == 0
    _check(paired.float().cpu().numpy(), ref["out"])
    _check(plain.float().cpu().numpy(), ref["out"])
    np.testing.assert_allclose(lse_p.cpu().numpy(), ref["lse"], atol=2e-3, rtol=1e-4)
