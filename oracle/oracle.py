"""CPU oracle for the Spark-H3 hot path.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline
leg of ``bench.py`` import this module, and only as the checker; the product path never
calls it.

Integer outputs (route indices, packed words) come from ``spark_oracle.c``, which fixes
the arithmetic order shared with the CUDA kernels.  Floating-point outputs (anchor,
summaries, attention) are restated here in numpy with float64 accumulation and the same
storage roundings as the reference:

* anchor        h3_sparse_attention/sol_numerator_virtual_q.py:268-302
* summaries     h3_sparse_attention/sol_numerator_virtual_q.py:93-135 (_summaries)
* attention     tests/test_spark_installer.py:559-570 (explicit exact/summary softmax) with
                the exact-block rule of sol_attn/sm90/mainloop.py:590-667 and the dense
                suffix of h3_sparse_attention/spark_integration.py:1251-1261
"""
from __future__ import annotations

import ctypes
import hashlib
import math
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_build" / "libsparkoracle.so"
LOG2E = 1.4426950408889634
LN2 = 0.6931471805599453


def build() -> Path:
    """Compile the C restatement (gcc, no contraction of multiply-adds)."""
    LIB_PATH.parent.mkdir(parents=True, exist_ok=True)
    sources = [HERE / "spark_oracle.c", HERE / "reblock_oracle.c"]
    flags = ["-O2", "-ffp-contract=off", "-fno-fast-math", "-fopenmp", "-shared", "-fPIC"]
    stamp = LIB_PATH.with_suffix(".stamp")
    digest = hashlib.sha256(" ".join(flags).encode() + b"".join(src.read_bytes() for src in sources)).hexdigest()
    if LIB_PATH.exists() and stamp.exists() and stamp.read_text() == digest:
        return LIB_PATH
    tmp = LIB_PATH.with_suffix(f".{os.getpid()}.tmp")
    subprocess.check_call(["gcc", *flags, "-o", str(tmp), *map(str, sources), "-lm"])
    os.replace(tmp, LIB_PATH)
    stamp.write_text(digest)
    return LIB_PATH


_LIB = None


def _lib():
    global _LIB
    if _LIB is None:
        lib = ctypes.CDLL(str(build()))
        f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
        i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
        vp = ctypes.c_void_p
        ci, cf, ci64 = ctypes.c_int, ctypes.c_float, ctypes.c_int64
        lib.orc_block_means.argtypes = [vp, ci, ci, ci, ci, ci, ci, f32p]
        lib.orc_round_bf16.argtypes = [f32p, ci64]
        lib.orc_anchor.argtypes = [f32p, ci, ci, ci, ci, ci, ci, f32p]
        lib.orc_scores.argtypes = [f32p, f32p, ci, ci, ci, ci, ci, ci, cf, f32p]
        lib.orc_topk.argtypes = [f32p, ci64, ci, ci, ci, i32p, i32p]
        lib.orc_topk_head_budgets.argtypes = [f32p, ci64, ci, ci, i32p, ci, ci, i32p, i32p]
        for fn in (lib.orc_block_means, lib.orc_round_bf16, lib.orc_anchor, lib.orc_scores, lib.orc_topk,
                   lib.orc_topk_head_budgets):
            fn.restype = None
        u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
        lib.orc_rb_norms.argtypes = [u16p, ci64, ci, f32p]
        lib.orc_rb_norms.restype = None
        lib.orc_rb_tree.argtypes = [u16p, ci, ci, ci, i32p, i32p, i32p]
        lib.orc_rb_tree.restype = ci
        lib.orc_rb_tree_proxy.argtypes = [u16p, ci, ci, ci, i32p, i32p, ci, ci, ctypes.c_void_p, i32p]
        lib.orc_rb_tree_proxy.restype = ci
        _LIB = lib
    return _LIB


# ------------------------------------------------------------------ bf16 helpers
def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bfloat16 bit patterns (NaN kept quiet)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7F800000) == 0x7F800000
    nan &= (u & 0x007FFFFF) != 0
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) & 0xFFFF
    out = np.where(nan, ((u >> 16) | 0x40) & 0xFFFF, rounded)
    return out.astype(np.uint16)


def round_bf16(x: np.ndarray) -> np.ndarray:
    return bf16_bits_to_f32(f32_to_bf16_bits(np.asarray(x, dtype=np.float32)))


class Tensor:
    """A host tensor in its storage dtype: float32 values or bfloat16 bit patterns."""

    def __init__(self, data: np.ndarray, dtype: str):
        if dtype not in ("float32", "bfloat16"):
            raise ValueError("dtype must be float32 or bfloat16")
        want = np.uint16 if dtype == "bfloat16" else np.float32
        self.data = np.ascontiguousarray(data, dtype=want)
        self.dtype = dtype

    @property
    def shape(self):
        return self.data.shape

    def float(self) -> np.ndarray:
        return bf16_bits_to_f32(self.data) if self.dtype == "bfloat16" else self.data

    @property
    def code(self) -> int:
        return 1 if self.dtype == "bfloat16" else 0


def store(x: np.ndarray, dtype: str) -> np.ndarray:
    """Round float values to a storage dtype and return them as float32."""
    x = np.asarray(x, dtype=np.float32)
    return round_bf16(x) if dtype == "bfloat16" else x


# --------------------------------------------------------------- integer path
def block_means(x: Tensor, block: int) -> np.ndarray:
    B, T, H, D = x.shape
    nb = -(-T // block)
    out = np.empty((B, nb, H, D), dtype=np.float32)
    _lib().orc_block_means(x.data.ctypes.data, x.code, B, T, H, D, block, out)
    return out


def key_means(k: Tensor, block: int) -> np.ndarray:
    """Key block means stored at the key precision (returned as float32)."""
    kc = block_means(k, block)
    return store(kc, k.dtype)


def anchor(qc: np.ndarray, block: int, prefix_blocks: int, dtype: str) -> np.ndarray:
    B, NB, H, D = qc.shape
    out = np.empty((B, H, D), dtype=np.float32)
    _lib().orc_anchor(np.ascontiguousarray(qc), B, NB, H, D, block, prefix_blocks, out)
    return store(out, dtype)


def scale_log2(D: int) -> float:
    return float(np.float32(D ** -0.5 * LOG2E))


def scores(qc: np.ndarray, kc: np.ndarray, query_blocks: int, candidates: int) -> np.ndarray:
    B, NB, H, D = qc.shape
    out = np.empty((B, query_blocks, H, candidates), dtype=np.float32)
    _lib().orc_scores(np.ascontiguousarray(qc), np.ascontiguousarray(kc, dtype=np.float32), B, query_blocks,
                      NB, H, D, candidates, scale_log2(D), out)
    return out


def topk(score: np.ndarray, k: int, total_blocks: int) -> tuple[np.ndarray, np.ndarray]:
    """Ascending top-k indices [B, QB, H, k] and packed words [B, QB, H, ceil(NB/32)]."""
    B, QB, H, C = score.shape
    words = -(-total_blocks // 32)
    rows = B * QB * H
    idx = np.empty((rows, k), dtype=np.int32)
    packed = np.empty((rows, words), dtype=np.int32)
    _lib().orc_topk(np.ascontiguousarray(score), rows, C, k, words, idx, packed)
    return idx.reshape(B, QB, H, k), packed.reshape(B, QB, H, words)


def topk_head_budgets(score: np.ndarray, budgets, total_blocks: int, width: int | None = None):
    """Per-head budgets (head_budget.py:7-19): row (b, q, h) keeps the budgets[h] largest
    scores, ties to the lower index.  Returns indices [B, QB, H, width] (ascending, -1 past
    the row's budget; width defaults to the largest budget) and packed words."""
    B, QB, H, C = score.shape
    budgets = np.ascontiguousarray(np.asarray(budgets, dtype=np.int32).reshape(H))
    if width is None:
        width = max(1, int(np.clip(budgets, 0, C).max()))
    words = -(-total_blocks // 32)
    rows = B * QB * H
    idx = np.empty((rows, width), dtype=np.int32)
    packed = np.empty((rows, words), dtype=np.int32)
    _lib().orc_topk_head_budgets(np.ascontiguousarray(score), rows, H, C, budgets, width, words, idx, packed)
    return idx.reshape(B, QB, H, width), packed.reshape(B, QB, H, words)


def target_topk(ratio: float, candidates: int) -> int:
    """max(1, round(ratio * candidates)) capped at candidates (sol_topk_cutoff.py:342)."""
    return min(max(1, round(ratio * candidates)), candidates)


# ------------------------------------------------------------ float restatements
def summaries(a: np.ndarray, k: Tensor, v: Tensor, block: int, *, weighted_kv: bool = True,
              mass_bias: bool = True, summary_math: str = "tensorcore",
              logmass_key: str = "stored") -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """AK, AV [B, H, NB, D] (stored precision) and LM [B, H, NB] for the global anchor
    (sol_numerator_virtual_q.py:93-193).  summary_math "tensorcore" rounds the
    probabilities to the K/V dtype before the weighted sums, "comfy_fp32" keeps them in
    fp32; logmass_key "stored" takes the LM shift from the stored key, "pre_round" from the
    unrounded mean."""
    B, T, H, D = k.shape
    nb = -(-T // block)
    kf, vf = k.float(), v.float()
    a64 = a.astype(np.float64)
    scale = D ** -0.5
    ak = np.empty((B, H, nb, D), dtype=np.float32)
    av = np.empty_like(ak)
    lm = np.empty((B, H, nb), dtype=np.float32)
    full = T // block
    # Runs of up to 64 whole blocks are evaluated together ([B, J, r, H, D] slabs); a partial
    # final block is its own run.  Every block's arithmetic is the per-block formula.
    runs = [(j, min(full, j + 64)) for j in range(0, full, 64)] + ([(full, nb)] if nb > full else [])
    for j0, j1 in runs:
        r = min(block, T - j0 * block)
        kk = kf[:, j0 * block:min(T, j1 * block)].astype(np.float64).reshape(B, j1 - j0, r, H, D)
        vv = vf[:, j0 * block:min(T, j1 * block)].astype(np.float64).reshape(B, j1 - j0, r, H, D)
        if weighted_kv or mass_bias:
            logits = np.einsum("bhd,bjrhd->bhjr", a64, kk) * scale * LOG2E
            mx = logits.max(-1, keepdims=True)
            p = np.exp2(logits - mx)
            den = p.sum(-1)                                   # [B, H, J]
        if weighted_kv:
            w = (p if summary_math == "comfy_fp32" else store(p, k.dtype)).astype(np.float64)
            key = np.einsum("bhjr,bjrhd->bhjd", w, kk) / den[..., None]
            val = np.einsum("bhjr,bjrhd->bhjd", w, vv) / den[..., None]
        else:
            key = kk.mean(2).transpose(0, 2, 1, 3)
            val = vv.mean(2).transpose(0, 2, 1, 3)
        ak[:, :, j0:j1] = store(key, k.dtype)
        av[:, :, j0:j1] = store(val, v.dtype)
        if mass_bias:
            shift_key = key if logmass_key == "pre_round" else ak[:, :, j0:j1].astype(np.float64)
            shift = np.einsum("bhd,bhjd->bhj", a64, shift_key) * scale
            lm[:, :, j0:j1] = (mx[..., 0] + np.log2(den)) * LN2 - shift
        else:
            lm[:, :, j0:j1] = math.log(r)
    return ak, av, lm


def summaries8(a: np.ndarray, k: Tensor, v: Tensor, *, weighted_kv: bool = True, mass_bias: bool = True,
               logmass_key: str = "stored") -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """Eight-key anchor summaries of the block8x8 tail (sol_numerator_virtual_q.py:193-242):
    fp32 probabilities, keys and values stored at the K/V precision, LM from the stored key
    (or the fp32 mean with logmass_key "pre_round")."""
    B, T, H, D = k.shape
    n8 = -(-T // 8)
    kf, vf = k.float().astype(np.float64), v.float().astype(np.float64)
    scale = D ** -0.5
    ak = np.empty((B, H, n8, D), dtype=np.float32)
    av = np.empty_like(ak)
    lm = np.empty((B, H, n8), dtype=np.float32)
    for g in range(n8):
        kk, vv = kf[:, 8 * g:8 * g + 8], vf[:, 8 * g:8 * g + 8]
        count = kk.shape[1]
        logits = np.einsum("bhd,brhd->bhr", a.astype(np.float64), kk) * scale * LOG2E
        mx = logits.max(-1)
        p = np.exp2(logits - mx[..., None])
        den = np.maximum(p.sum(-1), 1e-30)
        if weighted_kv:
            key = np.einsum("bhr,brhd->bhd", p, kk) / den[..., None]
            val = np.einsum("bhr,brhd->bhd", p, vv) / den[..., None]
        else:
            key, val = kk.mean(1), vv.mean(1)
        ak[:, :, g] = store(key, k.dtype)
        av[:, :, g] = store(val, v.dtype)
        if mass_bias:
            shift_key = key if logmass_key == "pre_round" else ak[:, :, g].astype(np.float64)
            lm[:, :, g] = (mx + np.log2(den)) * LN2 - np.einsum("bhd,bhd->bh", a.astype(np.float64), shift_key) * scale
        else:
            lm[:, :, g] = math.log(count)
    return ak, av, lm


def tail_merge(q: Tensor, exact_out: np.ndarray, exact_lse: np.ndarray, ak: np.ndarray, av: np.ndarray,
               lm: np.ndarray, packed: np.ndarray, *, block: int, entry_tokens: int, group_tokens: int,
               query_tokens: int, sink_first: int, sink_last: int, local_radius: int = -1,
               heads: list[int] | None = None) -> tuple[np.ndarray, np.ndarray]:
    """Pooled-tail merge (sol_numerator_virtual_q.py:415-499): per query group, the mean query
    (fp32, stored at Q's precision) attends the summary entries whose key block is not exact;
    rows blend that with their exact output by their LSE weights."""
    B, T, H, D = q.shape
    nb = -(-T // block)
    out, lse = exact_out.copy(), exact_lse.copy()
    qf = q.float()
    scale = D ** -0.5
    heads = list(range(H)) if heads is None else heads
    n_entries = ak.shape[2]
    entry_block = (np.arange(n_entries) * entry_tokens) // block
    for b in range(B):
        for h in heads:
            for g0 in range(0, query_tokens, group_tokens):
                rows = slice(g0, min(g0 + group_tokens, T))
                qb = g0 // block
                qmean = store(qf[b, rows, h].astype(np.float64).mean(0), q.dtype).astype(np.float64)
                exact = exact_blocks(packed[b, qb, h], qb, nb, sink_first, sink_last, local_radius)
                live = ~exact[entry_block]
                if live.any():
                    score = ak[b, h][live].astype(np.float64) @ qmean * scale + lm[b, h][live]
                    m = score.max()
                    p = np.exp(score - m)
                    tail = p @ av[b, h][live].astype(np.float64) / p.sum()
                    al = m + np.log(p.sum())
                else:
                    tail, al = np.zeros(D), -np.inf
                el = exact_lse[b, rows, h].astype(np.float64)
                mx = np.maximum(el, al)
                with np.errstate(invalid="ignore"):
                    we = np.where(np.isfinite(mx), np.exp(el - mx), 0.0)
                    wa = np.where(np.isfinite(mx), np.exp(al - mx), 0.0)
                tot = we + wa
                blend = (we[:, None] * exact_out[b, rows, h] + wa[:, None] * tail[None, :]) / np.maximum(tot, 1e-30)[:, None]
                out[b, rows, h] = blend.astype(np.float32)
                with np.errstate(divide="ignore"):
                    lse[b, rows, h] = np.where(tot > 0, mx + np.log(np.maximum(tot, 1e-300)), -np.inf).astype(np.float32)
    return out, lse


def exact_blocks(packed_row: np.ndarray, qb: int, nb: int, sink_first: int, sink_last: int,
                 local_radius: int) -> np.ndarray:
    """Boolean [nb]: key blocks evaluated exactly for routed query block qb."""
    kb = np.arange(nb)
    bits = (packed_row[kb >> 5].astype(np.int64) >> (kb & 31)) & 1
    exact = bits.astype(bool) | ((kb >= sink_first) & (kb < sink_last))
    if local_radius >= 0:
        exact |= np.abs(qb - kb) <= local_radius
    return exact


def sparse_attention(q: Tensor, k: Tensor, v: Tensor, block: int, packed: np.ndarray, ak: np.ndarray,
                     av: np.ndarray, lm: np.ndarray, query_tokens: int, sink_first: int, sink_last: int,
                     local_radius: int = -1, rows: slice | list[slice] | None = None,
                     heads: list[int] | None = None) -> tuple[np.ndarray, np.ndarray]:
    """Output [B, T, H, D] float32 (unrounded) and LSE [B, T, H] for the selected rows/heads.

    ``rows`` is one slice or a list of slices.  Rows outside them / heads outside ``heads``
    are left as NaN.
    """
    B, T, H, D = q.shape
    nb = -(-T // block)
    qf, kf, vf = (x.float() for x in (q, k, v))
    out = np.full((B, T, H, D), np.nan, dtype=np.float32)
    lse = np.full((B, T, H), np.nan, dtype=np.float32)
    spans = rows if isinstance(rows, list) else [rows or slice(0, T)]
    heads = list(range(H)) if heads is None else heads
    scale = D ** -0.5
    for b in range(B):
        for h in heads:
            kh = kf[b, :, h].astype(np.float64)
            vh = vf[b, :, h].astype(np.float64)
            # ak/av/lm None: routed rows see their exact blocks only (no summary columns)
            akh = ak[b, h].astype(np.float64) if ak is not None else np.zeros((nb, D))
            avh = av[b, h].astype(np.float64) if av is not None else np.zeros((nb, D))
            lmh = lm[b, h].astype(np.float64) if lm is not None else np.zeros(nb)
            for span in spans:
                r0, r1 = span.start or 0, min(T, span.stop if span.stop is not None else T)
                start = r0
                while start < r1:
                    if start < query_tokens:
                        qb = start // block
                        stop = min(r1, (qb + 1) * block, query_tokens)
                        exact = exact_blocks(packed[b, qb, h], qb, nb, sink_first, sink_last, local_radius)
                    else:
                        qb = -1
                        stop = r1
                        exact = np.ones(nb, dtype=bool)
                    tok = np.repeat(exact, block)[:T]
                    summ = ~exact if ak is not None else np.zeros(nb, dtype=bool)
                    keys = np.concatenate([kh[tok], akh[summ]])
                    vals = np.concatenate([vh[tok], avh[summ]])
                    qq = qf[b, start:stop, h].astype(np.float64)
                    logits = qq @ keys.T * scale
                    logits[:, int(tok.sum()):] += lmh[summ]
                    if logits.shape[1] == 0:  # nothing visible
                        out[b, start:stop, h] = 0.0
                        lse[b, start:stop, h] = -np.inf
                        start = stop
                        continue
                    mx = logits.max(-1, keepdims=True)
                    p = np.exp(logits - mx)
                    den = p.sum(-1, keepdims=True)
                    out[b, start:stop, h] = (p @ vals / den).astype(np.float32)
                    lse[b, start:stop, h] = (mx[:, 0] + np.log(den[:, 0])).astype(np.float32)
                    start = stop
    return out, lse


# ------------------------------------------------------------- full pipeline
def block_pairs(packed: np.ndarray, blocks: int, window: int = 64) -> np.ndarray:
    """Query-block pairs of sb_route_pair_blocks, restated for its test (a tile scheduling
    choice of this build with no reference counterpart).  Per (b, h), in block order, every
    unpaired block among the first `blocks` takes the unpaired block of the largest route
    overlap among the next `window` (ties: the nearer); blocks left without a partner are
    then paired with each other in order.  Returns [B, H, ceil(blocks / 2), 2] int32, -1 for
    the empty half of an odd count."""
    B, QB, H, words = packed.shape
    bits = np.unpackbits(np.ascontiguousarray(packed).view(np.uint8), axis=-1, bitorder="little").astype(bool)
    out = np.full((B, H, -(-blocks // 2), 2), -1, np.int32)
    for b in range(B):
        for h in range(H):
            rows = bits[b, :blocks, h]
            taken = np.zeros(blocks, bool)
            pairs, singles = [], []
            for a in range(blocks):
                if taken[a]:
                    continue
                taken[a] = True
                best, best_ov = -1, -1
                for c in range(a + 1, min(blocks, a + 1 + window)):
                    if taken[c]:
                        continue
                    ov = int(np.count_nonzero(rows[a] & rows[c]))
                    if ov > best_ov:
                        best, best_ov = c, ov
                if best < 0:
                    singles.append(a)
                else:
                    taken[best] = True
                    pairs.append((a, best))
            for i in range(0, len(singles), 2):
                pairs.append((singles[i], singles[i + 1] if i + 1 < len(singles) else -1))
            out[b, h] = np.asarray(pairs, np.int32)
    return out


def padded_tail(q: Tensor, video: int, query_tokens: int, block: int) -> Tensor:
    """Q with rows [video, query_tokens) replaced by the mean of the final partial video
    block's rows, fp32 mean rounded to Q's dtype (spark_integration.py:1173-1187)."""
    if query_tokens <= video:
        return q
    tail_start = (video // block) * block
    mean = q.float()[:, tail_start:video].astype(np.float64).mean(axis=1, keepdims=True).astype(np.float32)
    data = q.data.copy()
    if q.dtype == "bfloat16":
        data[:, video:query_tokens] = f32_to_bf16_bits(mean)
    else:
        data[:, video:query_tokens] = mean
    return Tensor(data, q.dtype)


def spark_layer(q: Tensor, k: Tensor, v: Tensor, *, block: int, topk_ratio: float, video_tokens: int | None = None,
                anchor_dtype: str | None = None, local_radius: int = -1, weighted_kv: bool = True,
                mass_bias: bool = True, attention: bool = True, rows: slice | None = None,
                heads: list[int] | None = None, tail_mode: str = "dense", tail_granularity: str = "query",
                summary_math: str = "tensorcore", logmass_key: str = "stored", head_budgets=None) -> dict:
    """Route, summaries and (optionally) attention of one Spark layer, as the CUDA path does.

    head_budgets (one int per head): the per-head Top-K of head_budget.py:7-19 replaces the
    fixed budget, and every key block past the candidates is exact when there is a context
    suffix or a partial video block (head_budget.py:16-18).

    tail_mode "pad" (spark_integration.py:72-91, 935-938, 1173-1187, 1238-1260): the query
    prefix extends over the partial final video block, whose missing rows are filled with
    the mean of its video rows for the route; every row from the video end on is dense."""
    B, T, H, D = q.shape
    video = T if video_tokens is None else video_tokens
    nb = -(-T // block)
    if tail_mode == "dense":
        query_tokens = (video // block) * block
    elif tail_mode == "legacy_full":  # spark_integration.py:925-933, 1221-1262
        query_tokens = -(-video // block) * block
        if query_tokens > T:
            raise NotImplementedError("the final query block must be filled by the sequence")
    elif tail_mode == "pad":
        query_tokens = -(-video // block) * block
        if query_tokens > T:
            raise ValueError("the packed suffix is too short to pad the final video query block")
    else:
        raise ValueError("tail_mode must be 'dense', 'pad' or 'legacy_full'")
    query_blocks = query_tokens // block
    candidates = video // block
    sink_first = video // block
    sink_last = -(-T // block) if T > video else sink_first
    qc = block_means(padded_tail(q, video, query_tokens, block) if tail_mode == "pad" else q, block)
    kc = key_means(k, block)
    a = anchor(qc, block, candidates, anchor_dtype or q.dtype)
    sc = scores(qc, kc, query_blocks, candidates)
    kk = target_topk(topk_ratio, candidates)
    if head_budgets is None:
        idx, packed = topk(sc, kk, nb)
    else:
        idx, packed = topk_head_budgets(sc, head_budgets, nb, width=kk)
        if T > video or video % block:
            sink_first, sink_last = candidates, nb
    result = dict(qc=qc, kc=kc, anchor=a, scores=sc, indices=idx, packed=packed, topk=kk,
                  query_tokens=query_tokens, sink_first=sink_first, sink_last=sink_last)
    ak, av, lm = summaries(a, k, v, block, weighted_kv=weighted_kv, mass_bias=mass_bias,
                           summary_math=summary_math, logmass_key=logmass_key)
    result.update(ak=ak, av=av, lm=lm)
    if attention and tail_granularity != "query":
        # Exact keys only, then the pooled tail merged in (sol_numerator_virtual_q.py:655-660).
        if tail_mode != "dense":
            raise NotImplementedError("the oracle's pooled tails use tail_mode 'dense'")
        eo, el = sparse_attention(q, k, v, block, packed, None, None, None, query_tokens, sink_first, sink_last,
                                  local_radius, rows=rows, heads=heads)
        if tail_granularity == "block":
            tak, tav, tlm, entry, group = ak, av, lm, block, block
        else:
            tak, tav, tlm = summaries8(a, k, v, weighted_kv=weighted_kv, mass_bias=mass_bias, logmass_key=logmass_key)
            entry, group = 8, 8
        out, lse = tail_merge(q, np.nan_to_num(eo), el, tak, tav, tlm, packed, block=block, entry_tokens=entry,
                              group_tokens=group, query_tokens=query_tokens, sink_first=sink_first,
                              sink_last=sink_last, local_radius=local_radius, heads=heads)
        result.update(out=out, lse=lse)
    elif attention:
        out, lse = sparse_attention(q, k, v, block, packed, ak, av, lm, query_tokens, sink_first, sink_last,
                                    local_radius, rows=rows, heads=heads)
        if query_tokens > video:
            r0 = max(video, (rows.start or 0) if rows else 0)
            r1 = min(query_tokens, rows.stop if rows and rows.stop is not None else T)
            if r0 < r1:
                dense, dense_lse = sparse_attention(q, k, v, block, packed, ak, av, lm, 0, sink_first, sink_last,
                                                    local_radius, rows=slice(r0, r1), heads=heads)
                out[:, r0:r1], lse[:, r0:r1] = dense[:, r0:r1], dense_lse[:, r0:r1]
        result.update(out=out, lse=lse)
    return result


# ------------------------------------------------------------- reblock (landmark tree v2)
def hilbert_distances_3d(coords: np.ndarray, bits: int) -> np.ndarray:
    """Skilling transpose -> Hilbert index of integer [N, 3] coordinates
    (h3_sparse_attention/mahalanobis_kmeans.py:11-45)."""
    x = coords.astype(np.int64).copy()
    q = 1 << (bits - 1)
    while q > 1:
        mask = q - 1
        for axis in range(3):
            high = (x[:, axis] & q) != 0
            x[high, 0] ^= mask
            low = ~high
            swap = (x[low, 0] ^ x[low, axis]) & mask
            x[low, 0] ^= swap
            x[low, axis] ^= swap
        q >>= 1
    x[:, 1] ^= x[:, 0]
    x[:, 2] ^= x[:, 1]
    t = np.zeros(len(x), dtype=np.int64)
    q = 1 << (bits - 1)
    while q > 1:
        t[(x[:, 2] & q) != 0] ^= q - 1
        q >>= 1
    x ^= t[:, None]
    out = np.zeros(len(x), dtype=np.int64)
    for bit in range(bits - 1, -1, -1):
        for axis in range(3):
            out = (out << 1) | ((x[:, axis] >> bit) & 1)
    return out


def initial_order(grid, name: str = "flat") -> np.ndarray:
    """Root token order (landmark_initial_order.py:44-62)."""
    T_, H_, W_ = (int(g) for g in grid)
    ids = np.arange(T_ * H_ * W_, dtype=np.int64)
    if name == "flat":
        return ids
    t, h, w = ids // (H_ * W_), (ids // W_) % H_, ids % W_
    if name == "tile_t4h4w4":
        tile = ((t // 4) * ((H_ + 3) // 4) + h // 4) * ((W_ + 3) // 4) + w // 4
        return np.argsort(tile * 64 + (t % 4) * 16 + (h % 4) * 4 + w % 4, kind="stable")
    axes = dict(t=t, h=h, w=w)
    coords = np.stack([axes[a] for a in name[8:]], axis=-1)
    bits = max(1, (max(T_, H_, W_) - 1).bit_length())
    return np.argsort(hilbert_distances_3d(coords, bits), kind="stable")


def hilbert_midpoint_samples(grid, count: int) -> np.ndarray:
    """count metric samples, uniformly spaced along the 3-D Hilbert order
    (mahalanobis_kmeans.py:48-96)."""
    order = initial_order(grid, "hilbert_thw")
    n = len(order)
    count = min(max(1, int(count)), n)
    pos = np.floor((np.arange(count, dtype=np.float64) + 0.5) * n / count).astype(np.int64)
    return order[np.minimum(pos, n - 1)]


def metric_factors(q: Tensor, k: Tensor, samples: np.ndarray, video: int, ridge: float = 1e-3) -> np.ndarray:
    """Ridged non-centred second moments of the sampled Q and K rows and their Cholesky
    factors (mahalanobis_kmeans.py:309-388, landmark_direction.py:60-104), in float64:
    returns L [2*B*H, D, D], rows [0, BH) = chol(M2(Q)) (applied to K) and
    [BH, 2BH) = chol(M2(K)) (applied to Q)."""
    B, T, H, D = q.shape
    out = []
    for src in (q, k):
        x = src.float()[:, :video][:, samples].astype(np.float64)  # [B, S, H, D]
        for b in range(B):
            for h in range(H):
                s = x[b, :, h]
                m = s.T @ s / len(samples)
                m = 0.5 * (m + m.T)
                m[np.diag_indices(D)] += ridge * np.trace(m) / D
                out.append(np.linalg.cholesky(m))
    return np.stack(out)


def reblock_features(q: Tensor, k: Tensor, factors: np.ndarray, video: int) -> np.ndarray:
    """[K . Lq ; Q . Lk] of bf16 operands, accumulated exactly and stored bf16
    (spark_integration.py:561-585): uint16 bf16 bits [2*B*H, video, D]."""
    B, T, H, D = q.shape
    rows = []
    lf = round_bf16(np.asarray(factors, dtype=np.float32))
    for side, src in enumerate((k, q)):
        x = src.float()[:, :video]
        for b in range(B):
            for h in range(H):
                r = side * B * H + b * H + h
                prod = x[b, :, h].astype(np.float64) @ lf[r].astype(np.float64)
                rows.append(f32_to_bf16_bits(prod.astype(np.float32)))
    return np.stack(rows)


def hierarchy_schedule(split_budgets) -> np.ndarray:
    """Encode a hierarchy's per-round (leaves, child budgets) table for orc_rb_tree."""
    words = [len(split_budgets)]
    for level in split_budgets:
        words.append(len(level))
        for leaves, budgets in level:
            words += [leaves, len(budgets), *budgets]
    return np.asarray(words, dtype=np.int32)


def remainder_ids(features_bits: np.ndarray) -> np.ndarray:
    """The protected remainder of bf16 features [rows, N, D] (landmark_tree_clustering.py:56-82):
    per row the N mod 64 ids of largest squared norm (reblock_oracle.c's canonical sum), equal
    norms to the lower id, ascending; int32 [rows, N mod 64]."""
    x = np.ascontiguousarray(features_bits, dtype=np.uint16)
    rows, n, d = x.shape
    rem = n % 64
    out = np.zeros((rows, rem), dtype=np.int32)
    norms = np.empty(n, dtype=np.float32)
    for r in range(rows):
        _lib().orc_rb_norms(x[r], n, d, norms)
        order = np.lexsort((np.arange(n), -norms.astype(np.float64)))  # largest first, lower id first
        out[r] = np.sort(order[:rem])
    return out


def reblock_tree(features_bits: np.ndarray, grid, split_budgets, order: str = "flat", *, proxy_iterations: int = 2,
                 seed_rule: str = "farthest_pair", excluded=None) -> tuple[np.ndarray, np.ndarray]:
    """Landmark-tree-v2 permutation of bf16 features [rows, N, D] (reblock_oracle.c), with the
    proxy controls of landmark_v2_terminal.py:43-50 (mean updates) and optionally the caller's
    protected remainder `excluded` [rows, N mod 64]: returns (permutation, inverse) int64
    [rows, N]."""
    if seed_rule not in ("farthest_pair", "endpoint_order"):
        raise ValueError("seed_rule must be farthest_pair or endpoint_order")
    x = np.ascontiguousarray(features_bits, dtype=np.uint16)
    rows, n, d = x.shape
    root = np.ascontiguousarray(initial_order(grid, order), dtype=np.int32)
    perm = np.empty((rows, n), dtype=np.int32)
    frozen = None if excluded is None else np.ascontiguousarray(excluded, dtype=np.int32)
    if frozen is not None and frozen.shape != (rows, n % 64):
        raise ValueError(f"excluded must have shape {(rows, n % 64)}")
    rc = _lib().orc_rb_tree_proxy(x, rows, n, d, root, hierarchy_schedule(split_budgets), proxy_iterations,
                                  int(seed_rule == "endpoint_order"),
                                  None if frozen is None else frozen.ctypes.data, perm)
    if rc != 0:
        raise RuntimeError(f"orc_rb_tree failed ({rc})")
    inverse = np.empty_like(perm)
    np.put_along_axis(inverse, perm, np.broadcast_to(np.arange(n, dtype=np.int32), perm.shape), axis=1)
    return perm.astype(np.int64), inverse.astype(np.int64)
