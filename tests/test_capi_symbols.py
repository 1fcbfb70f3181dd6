"""The C-ABI library loads on a CPU-only host and exports every entry point the header
declares, with the ctypes binding covering exactly those names; argument validation runs
before any CUDA call, so each rejected argument and its message are checked here too (no
compute calls)."""
import ctypes
import re
from pathlib import Path

from spark_h3_b200 import _build, _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "spark_h3_b200.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(sb_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_boundary():
    names = declared_functions()
    for required in ("sb_pool_queries", "sb_query_anchor", "sb_pool_keys_summaries", "sb_route_topk",
                     "sb_sparse_attention", "sb_headwise_permute", "sb_last_error"):
        assert required in names


def test_library_exports_every_declared_symbol():
    path = _build.build()
    lib = ctypes.CDLL(str(path))
    missing = [name for name in declared_functions() if not hasattr(lib, name)]
    assert not missing, missing


def test_ctypes_binding_matches_header():
    assert sorted(_lib.SIGNATURES) == declared_functions()


def test_version_and_error_calls_need_no_gpu():
    lib = _lib.load()
    assert lib.sb_version() >= 100
    assert isinstance(lib.sb_last_error(), bytes)


def test_invalid_arguments_are_rejected_before_any_launch():
    lib = _lib.load()
    # A null query pointer is an argument error (no device touched).
    rc = lib.sb_pool_queries(None, 1, 1, 128, 1, 128, 128, None, None)
    assert rc == -1
    assert b"null" in lib.sb_last_error()
    rc = lib.sb_route_topk(None, None, 1, 1, 1, 1, 1, 128, 1, 1, 1.0, None, None, None, None)
    assert rc == -1
    rc = lib.sb_headwise_permute(None, None, None, 4, 1, 1, 1, 128, 2, 1, None)
    assert rc == -1


# A valid routed call at block 64 (2048 tokens, 2 heads), then one argument changed per case.
# The pointers are fake but non-null and 16-byte aligned: validation never dereferences them
# and every case is rejected before the first CUDA call.
_P = 0x10000
_VALID = dict(q=_P, k=_P, v=_P, dtype=1, B=1, T=2048, H=2, D=128, block=64, packed=_P, QB=32, ak=_P, av=_P,
              lm=_P, query_tokens=2048, sink_first=32, sink_last=32, local_radius=-1, out=_P, lse=None,
              stream=None)
_ATTENTION_CASES = [
    (dict(q=None), b"null Q/K/V/out"),
    (dict(out=None), b"null Q/K/V/out"),
    (dict(dtype=7), b"bad dtype"),
    (dict(H=0), b"B, T, H must be positive"),
    (dict(D=96), b"head dim must be 64 or 128, got 96"),
    (dict(block=32), b"block must be 64 or 128, got 32"),
    (dict(T=(1 << 22) + 64, query_tokens=0), b"at most 4194304 tokens"),
    (dict(query_tokens=100), b"query_tokens must be a block multiple"),
    (dict(query_tokens=2112), b"query_tokens must be a block multiple"),
    (dict(packed=None), b"routed queries need the route"),
    (dict(av=None), b"pass all of AK, AV and LM, or none"),
    (dict(QB=5), b"QB (5) must lie in [32, 32]"),
    (dict(sink_first=5, sink_last=3), b"sink range [5, 3) is outside [0, 32]"),
    (dict(local_radius=-2), b"local_radius must be >= -1"),
    (dict(q=_P + 8), b"16-byte aligned"),
]


def test_sparse_attention_rejects_each_bad_argument_with_its_message():
    import pytest

    lib = _lib.load()
    order = ("q", "k", "v", "dtype", "B", "T", "H", "D", "block", "packed", "QB", "ak", "av", "lm",
             "query_tokens", "sink_first", "sink_last", "local_radius", "out", "lse", "stream")
    for change, message in _ATTENTION_CASES:
        args = {**_VALID, **change}
        rc = lib.sb_sparse_attention(*(args[name] for name in order))
        assert rc == -1, change
        assert message in lib.sb_last_error(), (change, lib.sb_last_error())
    with pytest.raises(_lib.SparkKernelError, match="head dim must be 64 or 128"):
        _lib.call("sb_sparse_attention", *({**_VALID, "D": 32}[name] for name in order))


def test_tail_merge_and_summaries_reject_bad_arguments():
    lib = _lib.load()
    merge = dict(q=_P, ak=_P, av=_P, lm=_P, dtype=1, B=1, T=2048, H=2, D=128, entry=8, group=8, block=64,
                 packed=_P, QB=32, query_tokens=2048, sink_first=32, sink_last=32, local_radius=-1, out=_P, lse=_P,
                 stream=None)
    order = tuple(merge)
    for change, message in [(dict(group=64), b"both whole blocks or both 8 tokens"),
                            (dict(entry=64, group=8), b"both whole blocks or both 8 tokens"),
                            (dict(dtype=0), b"Q and the output must be bf16"),
                            (dict(block=96), b"block must be 64 or 128"),
                            (dict(query_tokens=100), b"query_tokens must be a block multiple"),
                            (dict(lse=None), b"null pointer")]:
        args = {**merge, **change}
        assert lib.sb_tail_merge(*(args[n] for n in order)) == -1, change
        assert message in lib.sb_last_error(), (change, lib.sb_last_error())
    summ = dict(k=_P, v=_P, anchor=_P, dtype=1, anchor_dtype=1, B=1, T=2048, H=2, D=128, block=64, weighted=1,
                mass=1, numerics=0, kc=_P, ak=_P, av=_P, lm=_P, stream=None)
    order = tuple(summ)
    for change, message in [(dict(numerics=4), b"unknown numerics flags 4"),
                            (dict(D=96), b"head dim must be 64 or 128"),
                            (dict(anchor=None), b"weighted summaries need the anchor"),
                            (dict(v=None), b"summaries need V"),
                            (dict(block=32), b"block must be 64 or 128")]:
        args = {**summ, **change}
        assert lib.sb_pool_keys_summaries(*(args[n] for n in order)) == -1, change
        assert message in lib.sb_last_error(), (change, lib.sb_last_error())


def test_route_entry_points_name_themselves_in_their_errors():
    lib = _lib.load()
    args = dict(qc=_P, kc=_P, dtype=1, B=1, QB=32, NB=32, H=2, D=128, candidates=32)
    order = tuple(args)
    base = [args[n] for n in order]
    # sb_route_topk(..., topk, scale, workspace, packed, indices, stream)
    assert lib.sb_route_topk(*base, 40, 1.0, _P, _P, None, None) == -1
    assert lib.sb_last_error().startswith(b"sb_route_topk: topk must lie in [1, candidates], got 40")
    assert lib.sb_route_topk_noalloc(*base, 0, 1.0, _P, None, None) == -1
    assert lib.sb_last_error().startswith(b"sb_route_topk_noalloc: topk must lie in [1, candidates], got 0")
    # sb_route_topk_head_budgets(..., head_topk, index_width, scale, workspace, packed, indices, stream)
    assert lib.sb_route_topk_head_budgets(*base, None, 3, 1.0, _P, _P, None, None) == -1
    assert lib.sb_last_error().startswith(b"sb_route_topk_head_budgets: null pointer")
    assert lib.sb_route_topk_head_budgets(*base, _P, 33, 1.0, _P, _P, _P, None) == -1
    assert lib.sb_last_error().startswith(b"sb_route_topk_head_budgets: index_width must lie in [1, candidates]")
    bad = {**args, "D": 96}
    assert lib.sb_route_topk_head_budgets(*(bad[n] for n in order), _P, 3, 1.0, _P, _P, None, None) == -1
    assert lib.sb_last_error().startswith(b"sb_route_topk_head_budgets: head dim must be 64 or 128")
