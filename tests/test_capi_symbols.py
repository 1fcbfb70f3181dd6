"""The C-ABI library loads on a CPU-only host and exports every entry point the header
declares, with the ctypes binding covering exactly those names (no compute calls)."""
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
