"""Production-size inputs and the reference's route at that size.

Config 1 is one Spark layer at N = 124,992 (grid 31 x 48 x 84), H = 32, D = 128, bf16,
top-k ratio 0.1.  The seeded Q/K/V come from spark_h3_b200.synthetic on the CPU (the torch
CPU generator, the same stream tests/golden/make_golden.py drew them from) and are checked
against the SHA-256 digests recorded in tests/golden/route_config1_b64.npz before use.

That fixture holds the reference's own fp32 route (spark_integration.py:94-175,
_sol_topk_policy_scores + _sol_topk_route_from_scores) at its block size, 64 (1953 blocks,
k = 195): per (query block, head) row a 64-bit digest of the selected set and the gap between
the k-th and (k+1)-th reference score, plus the full sets of 256 seeded sample rows.
"""
from __future__ import annotations

import hashlib
import json
from pathlib import Path

import numpy as np
import torch

from oracle import oracle
from spark_h3_b200.synthetic import make_qkv

FIXTURE = Path(__file__).resolve().parent / "golden" / "route_config1_b64.npz"
GRID, HEADS, DIM = (31, 48, 84), 32, 128
TOKENS = GRID[0] * GRID[1] * GRID[2]
# Rows of the fixture where the oracle's selection differs from the reference's (measured:
# one row, whose k-th and (k+1)-th reference scores are equal).
MAX_TIE_ROWS = 1


def fixture() -> dict:
    g = np.load(FIXTURE)
    out = {name: g[name] for name in g.files}
    out["meta"] = json.loads(str(g["meta"]))
    return out


def _digest(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().view(torch.int16).numpy().tobytes()).hexdigest()


def inputs(with_v: bool = True):
    """Config-1 Q, K (and V) on the CPU, bf16 [1, N, 32, 128], digest-checked."""
    fx = fixture()
    meta = fx["meta"]
    tensors = make_qkv(tuple(meta["grid"]), meta["heads"], meta["dim"], seed=meta["seed"], dtype=torch.bfloat16,
                       q_scale=meta["q_scale"], with_v=with_v)
    assert _digest(tensors[0]) == str(fx["q_digest"]), "config-1 Q generator drifted from the fixture"
    assert _digest(tensors[1]) == str(fx["k_digest"]), "config-1 K generator drifted from the fixture"
    return tensors


def host(t: torch.Tensor) -> oracle.Tensor:
    """A bf16 CPU tensor as the oracle's Tensor (no copy beyond contiguity)."""
    return oracle.Tensor(t.contiguous().view(torch.int16).numpy().view(np.uint16), "bfloat16")


def row_digests(indices: np.ndarray) -> np.ndarray:
    """uint64 per row: the first 8 bytes (little endian) of the SHA-256 of the row's ascending
    int32 indices (the fixture's digest)."""
    rows = np.ascontiguousarray(np.sort(indices.reshape(-1, indices.shape[-1]), axis=-1).astype("<i4"))
    return np.array([int.from_bytes(hashlib.sha256(r.tobytes()).digest()[:8], "little") for r in rows],
                    dtype=np.uint64)


def compare_with_reference(indices: np.ndarray, fx: dict) -> np.ndarray:
    """Checks a block-64 route's ascending indices [1, QB, H, k] against the reference's and
    returns the mask of differing rows.  Rows may differ only where the reference's own k-th
    and (k+1)-th fp32 scores are equal: torch.topk leaves the order of equal scores
    unspecified, and this build takes the lower block id (head_budget.py:11's stable order)."""
    assert indices.shape[-1] == int(fx["target"])
    differ = row_digests(indices) != fx["row_digest"]
    assert np.all(fx["gap"][differ] == 0.0), fx["gap"][differ]
    assert int(differ.sum()) <= MAX_TIE_ROWS, int(differ.sum())
    flat = indices.reshape(-1, indices.shape[-1])
    for row, ref in zip(fx["sample_rows"], fx["sample_sets"]):
        if not differ[row]:
            assert np.array_equal(flat[row], ref.astype(np.int32)), row
    return differ
