"""Tensor-level wrappers over the C ABI.  Every op runs on the GPU through
libsparkh3b200.so; a non-CUDA tensor is an error, never a fallback."""
from __future__ import annotations

import math

import torch

from . import _lib

LOG2E = 1.4426950408889634


def _dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.bfloat16:
        return _lib.BF16
    if t.dtype == torch.float32:
        return _lib.F32
    raise TypeError(f"spark_h3_b200 supports float32 and bfloat16 tensors, got {t.dtype}")


def _require_cuda(*tensors: torch.Tensor) -> torch.device:
    device = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("spark_h3_b200 kernels require CUDA tensors; there is no CPU path")
        if not t.is_contiguous():
            raise RuntimeError("spark_h3_b200 kernels require contiguous tensors")
        if device is None:
            device = t.device
        elif t.device != device:
            raise RuntimeError("all tensors must be on the same CUDA device")
    return device


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def scale_log2(head_dim: int) -> float:
    return float(torch.tensor(head_dim ** -0.5 * LOG2E, dtype=torch.float32))


def target_topk(topk_ratio: float, candidates: int) -> int:
    """max(1, round(ratio * candidates)), capped at the candidate count
    (h3_sparse_attention/sol_topk_cutoff.py:342, spark_integration.py:132)."""
    return min(max(1, round(topk_ratio * candidates)), candidates)


def pool_queries(q: torch.Tensor, block: int) -> torch.Tensor:
    device = _require_cuda(q)
    B, T, H, D = q.shape
    nb = math.ceil(T / block)
    qc = torch.empty((B, nb, H, D), device=device, dtype=torch.float32)
    with torch.cuda.device(device):
        _lib.call("sb_pool_queries", q.data_ptr(), _dtype_code(q), B, T, H, D, block, qc.data_ptr(), _stream(device))
    return qc


def query_anchor(qc: torch.Tensor, block: int, prefix_blocks: int, dtype: torch.dtype) -> torch.Tensor:
    device = _require_cuda(qc)
    B, NB, H, D = qc.shape
    anchor = torch.empty((B, H, D), device=device, dtype=dtype)
    with torch.cuda.device(device):
        _lib.call("sb_query_anchor", qc.data_ptr(), B, NB, H, D, block, prefix_blocks, anchor.data_ptr(),
                  _dtype_code(anchor), _stream(device))
    return anchor


def pool_keys_summaries(k: torch.Tensor, v: torch.Tensor | None, anchor: torch.Tensor | None, block: int, *,
                        weighted_kv: bool = True, mass_bias: bool = True, want_kc: bool = True,
                        want_summaries: bool = True, summary_math: str = "tensorcore",
                        logmass_key: str = "stored"):
    """Returns (kc, ak, av, lm); entries not requested are None.  summary_math and
    logmass_key are the reference's summary ablations (processor.py:61-68)."""
    device = _require_cuda(k, v, anchor)
    B, T, H, D = k.shape
    if summary_math not in ("tensorcore", "comfy_fp32") or logmass_key not in ("stored", "pre_round"):
        raise ValueError("invalid reweight summary numeric mode")
    if summary_math == "comfy_fp32" and k.dtype != torch.bfloat16:
        raise ValueError("comfy_fp32 summaries require BF16 K/V")
    numerics = (_lib.SUMMARY_FP32_WEIGHTS if summary_math == "comfy_fp32" else 0) | \
        (_lib.SUMMARY_PRE_ROUND_LOGMASS if logmass_key == "pre_round" else 0)
    nb = math.ceil(T / block)
    kc = torch.empty((B, nb, H, D), device=device, dtype=k.dtype) if want_kc else None
    ak = av = lm = None
    if want_summaries:
        if v is None or v.shape != k.shape or v.dtype != k.dtype:
            raise ValueError("summaries need V with the shape and dtype of K")
        ak = torch.empty((B, H, nb, D), device=device, dtype=k.dtype)
        av = torch.empty_like(ak)
        lm = torch.empty((B, H, nb), device=device, dtype=torch.float32)
    anchor_code = _dtype_code(anchor) if anchor is not None else _dtype_code(k)
    with torch.cuda.device(device):
        _lib.call("sb_pool_keys_summaries", k.data_ptr(), _ptr(v), _ptr(anchor), _dtype_code(k), anchor_code,
                  B, T, H, D, block, int(weighted_kv), int(mass_bias), numerics, _ptr(kc), _ptr(ak), _ptr(av),
                  _ptr(lm), _stream(device))
    return kc, ak, av, lm


def route_workspace_bytes(B: int, query_blocks: int, H: int, candidates: int) -> int:
    return int(_lib.load().sb_route_workspace_bytes(B, query_blocks, H, candidates))


def route_topk(qc: torch.Tensor, kc: torch.Tensor, query_blocks: int, candidates: int, topk: int, *,
               workspace: torch.Tensor | None = None, want_indices: bool = True,
               head_budgets: torch.Tensor | None = None):
    """Packed route [B, QB, H, ceil(NB/32)] int32 and ascending indices [B, QB, H, topk].

    With head_budgets (int32 [H] on the device; head_budget.py:7-19) head h keeps its own
    head_budgets[h] blocks, clamped to [0, candidates]; the index rows are then `topk` wide
    and padded with -1 past each row's budget."""
    device = _require_cuda(qc, kc, workspace, head_budgets)
    B, NB, H, D = qc.shape
    words = math.ceil(NB / 32)
    need = route_workspace_bytes(B, query_blocks, H, candidates)
    if workspace is None:
        workspace = torch.empty(need, device=device, dtype=torch.uint8)
    elif workspace.numel() * workspace.element_size() < need:
        raise ValueError(f"route workspace holds {workspace.numel() * workspace.element_size()} bytes, needs {need}")
    packed = torch.empty((B, query_blocks, H, words), device=device, dtype=torch.int32)
    indices = torch.empty((B, query_blocks, H, topk), device=device, dtype=torch.int32) if want_indices else None
    with torch.cuda.device(device):
        if head_budgets is None:
            _lib.call("sb_route_topk", qc.data_ptr(), kc.data_ptr(), _dtype_code(kc), B, query_blocks, NB, H, D,
                      candidates, topk, scale_log2(D), workspace.data_ptr(), packed.data_ptr(), _ptr(indices),
                      _stream(device))
        else:
            if head_budgets.dtype != torch.int32 or head_budgets.shape != (H,):
                raise ValueError(f"head_budgets must be int32 [{H}], got {head_budgets.dtype} {tuple(head_budgets.shape)}")
            _lib.call("sb_route_topk_head_budgets", qc.data_ptr(), kc.data_ptr(), _dtype_code(kc), B, query_blocks,
                      NB, H, D, candidates, head_budgets.data_ptr(), topk, scale_log2(D), workspace.data_ptr(),
                      packed.data_ptr(), _ptr(indices), _stream(device))
    return packed, indices


def _check_query_prefix(query_tokens: int, tokens: int, block: int) -> None:
    """The sparse query prefix ends on a query block (sol_numerator_virtual_q.py:755-756)."""
    if query_tokens % block or not 0 <= query_tokens <= tokens:
        raise ValueError("query_tokens must end at a physical query-block boundary")


PAIR_MAX_WORDS = 256  # sb_route_pair_blocks handles routes of up to 256 words (8192 candidate blocks)


def route_pairs(packed: torch.Tensor, blocks: int) -> torch.Tensor:
    """Query-block pairs [B, H, ceil(blocks/2), 2] int32 for the attention kernel's 128-row
    tiles (sb_route_pair_blocks): each of the first `blocks` routed blocks with the unpaired
    block of the largest route overlap among the next 64."""
    device = _require_cuda(packed)
    B, QB, H, words = packed.shape
    pairs = torch.empty((B, H, -(-blocks // 2), 2), device=device, dtype=torch.int32)
    with torch.cuda.device(device):
        lib = _lib.load()
        ws = torch.empty(int(lib.sb_route_pair_workspace_bytes(B, H, blocks)), device=device, dtype=torch.uint8)
        _lib.call("sb_route_pair_blocks", packed.data_ptr(), B, QB, H, words, blocks, ws.data_ptr(),
                  pairs.data_ptr(), _stream(device))
    return pairs


def sparse_attention(q, k, v, block: int, packed: torch.Tensor | None, ak, av, lm, *, query_tokens: int,
                     sink_first: int, sink_last: int, local_radius: int = -1, out: torch.Tensor | None = None,
                     want_lse: bool = False, pair_blocks: bool = True, pairs: torch.Tensor | None = None):
    """The fused sparse attention (sb_sparse_attention).  With 64-token blocks on the
    tensor-core kernel the routed query blocks are paired by route overlap first
    (route_pairs), unless pair_blocks is False; `pairs` passes precomputed pairs."""
    _check_query_prefix(query_tokens, q.shape[1], block)
    device = _require_cuda(q, k, v, packed, ak, av, lm, out)
    B, T, H, D = q.shape
    if k.shape != q.shape or v.shape != q.shape or k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError("Q, K and V must share shape and dtype")
    if out is None:
        out = torch.empty_like(q)
    lse = torch.empty((B, T, H), device=device, dtype=torch.float32) if want_lse else None
    QB = packed.shape[1] if packed is not None else 0
    routed = query_tokens // block
    if (pairs is None and pair_blocks and block == 64 and routed >= 2 and q.dtype == torch.bfloat16 and D == 128
            and packed.shape[-1] <= PAIR_MAX_WORDS):
        pairs = route_pairs(packed, routed)
    with torch.cuda.device(device):
        _lib.call("sb_sparse_attention_pairs", q.data_ptr(), k.data_ptr(), v.data_ptr(), _dtype_code(q), B, T, H,
                  D, block, _ptr(packed), QB, _ptr(ak), _ptr(av), _ptr(lm), query_tokens, sink_first, sink_last,
                  local_radius, _ptr(pairs), out.data_ptr(), _ptr(lse), _stream(device))
    return out, lse


def pooled_tail_attention(q, k, v, block: int, packed, ak, av, lm, anchor, *, query_tokens: int, sink_first: int,
                          sink_last: int, local_radius: int = -1, out: torch.Tensor | None = None,
                          tail_granularity: str = "query", weighted_kv: bool = True, mass_bias: bool = True,
                          logmass_key: str = "stored") -> torch.Tensor:
    """The attention step of a Spark layer for each tail granularity
    (sol_numerator_virtual_q.py:597-660): "query" attends the summaries row by row inside the
    fused kernel; "block" and "block8x8" run the exact keys only and merge a pooled tail."""
    if tail_granularity == "query":
        o, _ = sparse_attention(q, k, v, block, packed, ak, av, lm, query_tokens=query_tokens, sink_first=sink_first,
                                sink_last=sink_last, local_radius=local_radius, out=out)
        return o
    if tail_granularity not in ("block", "block8x8"):
        raise ValueError("tail_granularity must be 'query', 'block', or 'block8x8'")
    o, lse = sparse_attention(q, k, v, block, packed, None, None, None, query_tokens=query_tokens,
                              sink_first=sink_first, sink_last=sink_last, local_radius=local_radius, out=out,
                              want_lse=True)
    if tail_granularity == "block":
        tak, tav, tlm, entry, group = ak, av, lm, block, block
    else:
        tak, tav, tlm = tail_summaries8(k, v, anchor, weighted_kv=weighted_kv, mass_bias=mass_bias,
                                        logmass_key=logmass_key)
        entry, group = 8, 8
    return tail_merge(q, tak, tav, tlm, packed, o, lse, block=block, entry_tokens=entry, group_tokens=group,
                      query_tokens=query_tokens, sink_first=sink_first, sink_last=sink_last,
                      local_radius=local_radius)


def dense_rows_attention(q, k, v, row_lo: int, row_hi: int, out: torch.Tensor, *,
                         lse: torch.Tensor | None = None) -> torch.Tensor:
    """Dense attention of query rows [row_lo, row_hi) over every key, written into `out`
    (and `lse`) in place; other rows are untouched (sb_dense_rows_attention)."""
    device = _require_cuda(q, k, v, out, lse)
    B, T, H, D = q.shape
    if k.shape != q.shape or v.shape != q.shape or out.shape != q.shape or out.dtype != q.dtype:
        raise ValueError("Q, K, V and out must share shape and dtype")
    with torch.cuda.device(device):
        _lib.call("sb_dense_rows_attention", q.data_ptr(), k.data_ptr(), v.data_ptr(), _dtype_code(q), B, T, H, D,
                  row_lo, row_hi, out.data_ptr(), _ptr(lse), _stream(device))
    return out


def tail_summaries8(k: torch.Tensor, v: torch.Tensor, anchor: torch.Tensor, *, weighted_kv: bool = True,
                    mass_bias: bool = True, logmass_key: str = "stored"):
    """Eight-key anchor summaries (AK8, AV8 [B, H, ceil(T/8), 128] bf16, LM8 fp32) of the
    block8x8 tail (sb_tail_summaries8)."""
    device = _require_cuda(k, v, anchor)
    B, T, H, D = k.shape
    if k.dtype != torch.bfloat16 or v.dtype != torch.bfloat16 or v.shape != k.shape or D != 128:
        raise ValueError("eight-key summaries take bf16 K/V [B, T, H, 128]")
    n8 = math.ceil(T / 8)
    ak8 = torch.empty((B, H, n8, D), device=device, dtype=k.dtype)
    av8 = torch.empty_like(ak8)
    lm8 = torch.empty((B, H, n8), device=device, dtype=torch.float32)
    numerics = _lib.SUMMARY_PRE_ROUND_LOGMASS if logmass_key == "pre_round" else 0
    with torch.cuda.device(device):
        _lib.call("sb_tail_summaries8", k.data_ptr(), v.data_ptr(), anchor.data_ptr(), _dtype_code(k),
                  _dtype_code(anchor), B, T, H, D, int(weighted_kv), int(mass_bias), numerics, ak8.data_ptr(),
                  av8.data_ptr(), lm8.data_ptr(), _stream(device))
    return ak8, av8, lm8


def tail_merge(q, ak, av, lm, packed: torch.Tensor, out: torch.Tensor, lse: torch.Tensor, *, block: int,
               entry_tokens: int, group_tokens: int, query_tokens: int, sink_first: int, sink_last: int,
               local_radius: int = -1) -> torch.Tensor:
    """Merges the pooled tail into the exact-only output and LSE in place (sb_tail_merge)."""
    _check_query_prefix(query_tokens, q.shape[1], block)
    device = _require_cuda(q, ak, av, lm, packed, out, lse)
    B, T, H, D = q.shape
    with torch.cuda.device(device):
        _lib.call("sb_tail_merge", q.data_ptr(), ak.data_ptr(), av.data_ptr(), lm.data_ptr(), _dtype_code(q), B, T,
                  H, D, entry_tokens, group_tokens, block, packed.data_ptr(), packed.shape[1], query_tokens,
                  sink_first, sink_last, local_radius, out.data_ptr(), lse.data_ptr(), _stream(device))
    return out


def padded_query_means(q: torch.Tensor, qc: torch.Tensor, video_tokens: int, query_tokens: int,
                       block: int) -> torch.Tensor:
    """sol_video_tail_mode = "pad" (spark_integration.py:1173-1187): the rows that fill the
    final video query block take the mean of that block's video rows (fp32 mean, rounded to
    Q's dtype), so its query mean is pooled over the padded block.  Only that block's mean
    changes: it is pooled from a one-block copy and written into qc in place."""
    tail_start = (video_tokens // block) * block
    if query_tokens <= video_tokens:
        return qc
    tail = q[:, tail_start:query_tokens].clone()
    tail[:, video_tokens - tail_start:] = q[:, tail_start:video_tokens].mean(dim=1, keepdim=True,
                                                                             dtype=torch.float32).to(q.dtype)
    qc[:, tail_start // block] = pool_queries(tail.contiguous(), block)[:, 0]
    return qc


def sparse_query_tokens(total_tokens: int, video_tokens: int, block: int, tail_mode: str = "dense") -> int:
    """Query prefix evaluated sparsely (spark_integration.py:72-91): the complete video blocks
    ("dense": the partial final block joins the dense suffix), or every video block with the
    final one padded from the context that follows ("pad"), or every video block with the
    final one pooled over the real video and context rows it holds ("legacy_full", the
    reference's sol_legacy_full_query, spark_integration.py:925-933)."""
    if tail_mode == "dense":
        return min(total_tokens, (video_tokens // block) * block)
    if tail_mode == "legacy_full":
        full = math.ceil(video_tokens / block) * block
        if full > total_tokens:
            raise NotImplementedError("sol_legacy_full_query with a final query block that the sequence does not "
                                      "fill is not implemented on the B200 path")
        return full
    if tail_mode != "pad":
        raise ValueError("tail_mode must be 'dense' or 'pad'")
    padded = math.ceil(video_tokens / block) * block
    if padded > total_tokens:
        raise ValueError("the packed suffix is too short to pad the final video query block")
    return padded


def headwise_permute(x: torch.Tensor, permutation: torch.Tensor, video_tokens: int,
                     out: torch.Tensor | None = None) -> torch.Tensor:
    """dst[b, t, h] = x[b, perm[b, h, t], h] for t < video_tokens; identity after."""
    device = _require_cuda(x, permutation, out)
    B, T, H, D = x.shape
    if permutation.shape != (B, H, video_tokens):
        raise ValueError(f"permutation must have shape {(B, H, video_tokens)}, got {tuple(permutation.shape)}")
    if permutation.dtype not in (torch.int32, torch.int64):
        raise TypeError("permutation must be int32 or int64")
    if out is None:
        out = torch.empty_like(x)
    with torch.cuda.device(device):
        _lib.call("sb_headwise_permute", x.data_ptr(), out.data_ptr(), permutation.data_ptr(),
                  permutation.element_size(), B, T, H, D, x.element_size(), video_tokens, _stream(device))
    return out


def read_device_status(device: torch.device | None = None) -> int:
    """Site code of the last bounded wait that gave up (0 = none); clears it.  Syncs."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    with torch.cuda.device(device):
        status = _lib.load().sb_read_device_status(_stream(device))
    _lib.check(min(status, 0), "sb_read_device_status")
    return status


def spark_layer(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *, block: int = 128, topk_ratio: float = 0.1,
                video_tokens: int | None = None, anchor_dtype: torch.dtype | None = None, local_radius: int = -1,
                weighted_kv: bool = True, mass_bias: bool = True, workspace: torch.Tensor | None = None,
                out: torch.Tensor | None = None, return_route: bool = False, tail_mode: str = "dense",
                tail_granularity: str = "query", summary_math: str = "tensorcore", logmass_key: str = "stored",
                head_budgets: torch.Tensor | None = None):
    """One Spark sparse attention layer on BTHD tensors whose video prefix comes first.

    pool Q -> anchor -> pool K + summaries -> scores + Top-K -> sparse attention
    (rows past the sparse query prefix are attended densely by the same kernel).  With
    tail_mode "pad" the partial final video block is routed as a padded block and the context
    rows that padded it are then attended densely (sb_dense_rows_attention); "legacy_full"
    routes it with the mean of all its rows, video and context, and attends its context rows
    densely the same way.  tail_granularity
    "block" / "block8x8" replaces the per-row summary columns by a pooled tail per query block
    / per 8 rows, merged into the exact-keys-only output (sb_tail_merge).  head_budgets
    (int32 [H] on the device) gives each head its own Top-K budget (head_budget.py:7-19); the
    blocks past the candidates are then exact when there is a context suffix or a partial
    video block.
    """
    B, T, H, D = q.shape
    video = T if video_tokens is None else int(video_tokens)
    if not block <= video <= T:
        raise ValueError(f"video_tokens must lie in [{block}, {T}]")
    query_tokens = sparse_query_tokens(T, video, block, tail_mode)
    query_blocks = query_tokens // block
    candidates = video // block
    nb = math.ceil(T / block)
    sink_first = video // block
    sink_last = nb if T > video else sink_first
    topk = target_topk(topk_ratio, candidates)
    if head_budgets is not None and (T > video or video % block):
        sink_first, sink_last = candidates, nb
    qc = pool_queries(q, block)
    if tail_mode == "pad":
        qc = padded_query_means(q, qc, video, query_tokens, block)
    anchor = query_anchor(qc, block, candidates, anchor_dtype or q.dtype)
    kc, ak, av, lm = pool_keys_summaries(k, v, anchor, block, weighted_kv=weighted_kv, mass_bias=mass_bias,
                                         summary_math=summary_math, logmass_key=logmass_key)
    packed, indices = route_topk(qc, kc, query_blocks, candidates, topk, workspace=workspace,
                                 want_indices=return_route, head_budgets=head_budgets)
    o = pooled_tail_attention(q, k, v, block, packed, ak, av, lm, anchor, query_tokens=query_tokens,
                              sink_first=sink_first, sink_last=sink_last, local_radius=local_radius, out=out,
                              tail_granularity=tail_granularity, weighted_kv=weighted_kv, mass_bias=mass_bias,
                              logmass_key=logmass_key)
    if query_tokens > video:
        dense_rows_attention(q, k, v, video, query_tokens, o)
    if return_route:
        return o, dict(qc=qc, kc=kc, anchor=anchor, ak=ak, av=av, lm=lm, packed=packed, indices=indices,
                       topk=topk, query_tokens=query_tokens, sink_first=sink_first, sink_last=sink_last)
    return o


def spark_layer_streamed(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, out: torch.Tensor, *, chunks: int = 4,
                         device: torch.device | None = None, **layer_args) -> torch.Tensor:
    """spark_layer on pinned host BTHD tensors, streamed by head chunks.

    Every stage of the layer is independent per (batch, head), so the heads are split into
    `chunks` groups: while group c runs on the GPU, group c+1 is uploaded and group c-1's
    output is downloaded (strided host<->device copies on two copy streams, double-buffered
    device memory).  `out` is the pinned host output.  Results are identical to spark_layer
    on the whole tensors.  The call returns with the last download queued on the current
    stream (synchronise it, or an event on it, before reading `out`)."""
    for name, t in (("q", q), ("k", k), ("v", v), ("out", out)):
        if t.is_cuda or not t.is_pinned() or not t.is_contiguous():
            raise RuntimeError(f"spark_layer_streamed takes contiguous pinned host tensors; {name} is not")
    if q.shape != k.shape or q.shape != v.shape or out.shape != q.shape or len({t.dtype for t in (q, k, v, out)}) != 1:
        raise ValueError("q, k, v and out must share one BTHD shape and dtype")
    B, T, H, D = q.shape
    if chunks < 1 or H % chunks:
        raise ValueError(f"{H} heads do not split into {chunks} equal chunks")
    device = device or torch.device("cuda", torch.cuda.current_device())
    hc = H // chunks
    es = q.element_size()
    row, chunk_row = H * D * es, hc * D * es
    main = torch.cuda.current_stream(device)
    up, down = torch.cuda.Stream(device), torch.cuda.Stream(device)
    dev_in = [[torch.empty((B, T, hc, D), device=device, dtype=q.dtype) for _ in range(3)] for _ in range(2)]
    dev_out = [torch.empty((B, T, hc, D), device=device, dtype=q.dtype) for _ in range(2)]
    block = layer_args.get("block", 128)
    video = layer_args.get("video_tokens") or T
    ws = layer_args.pop("workspace", None)
    if ws is None:
        ws = torch.empty(route_workspace_bytes(B, video // block, hc, video // block), device=device, dtype=torch.uint8)
    computed = [None, None]
    downloaded = [None, None]
    with torch.cuda.device(device):
        start = torch.cuda.Event()
        start.record(main)
        for c in range(chunks):
            slot = c & 1
            up.wait_event(start)
            if computed[slot] is not None:  # the slot's inputs were consumed by chunk c-2
                up.wait_event(computed[slot])
            for src, dst in zip((q, k, v), dev_in[slot]):
                _lib.call("sb_memcpy2d", dst.data_ptr(), chunk_row, src.data_ptr() + c * chunk_row, row, chunk_row,
                          B * T, up.cuda_stream)
            uploaded = torch.cuda.Event()
            uploaded.record(up)
            main.wait_event(uploaded)
            if downloaded[slot] is not None:  # the slot's output was read back for chunk c-2
                main.wait_event(downloaded[slot])
            spark_layer(*dev_in[slot], out=dev_out[slot], workspace=ws, **layer_args)
            computed[slot] = torch.cuda.Event()
            computed[slot].record(main)
            down.wait_event(computed[slot])
            _lib.call("sb_memcpy2d", out.data_ptr() + c * chunk_row, row, dev_out[slot].data_ptr(), chunk_row,
                      chunk_row, B * T, down.cuda_stream)
            downloaded[slot] = torch.cuda.Event()
            downloaded[slot].record(down)
        for ev in downloaded:
            if ev is not None:
                main.wait_event(ev)
    for t in dev_in[0] + dev_in[1] + dev_out:
        t.record_stream(up)
        t.record_stream(down)
    return out
