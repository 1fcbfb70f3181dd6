"""ctypes binding of the C ABI declared in include/spark_h3_b200.h.

Loading fails loudly when the shared library is missing: there is no CPU or Python
fallback for any entry point.
"""
from __future__ import annotations

import ctypes
import threading

from . import _build

F32 = 0
BF16 = 1

_lock = threading.Lock()
_lib = None

_vp = ctypes.c_void_p
_i = ctypes.c_int
_f = ctypes.c_float
_i64 = ctypes.c_int64

# sb_pool_keys_summaries numerics flags (SB_SUMMARY_* in include/spark_h3_b200.h).
SUMMARY_PRE_ROUND_LOGMASS = 1
SUMMARY_FP32_WEIGHTS = 2

# name -> (restype, argtypes); mirrors include/spark_h3_b200.h exactly.
SIGNATURES = {
    "sb_version": (_i, []),
    "sb_last_error": (ctypes.c_char_p, []),
    "sb_read_device_status": (_i, [_vp]),
    "sb_pool_queries": (_i, [_vp, _i, _i, _i, _i, _i, _i, _vp, _vp]),
    "sb_query_anchor": (_i, [_vp, _i, _i, _i, _i, _i, _i, _vp, _i, _vp]),
    "sb_pool_keys_summaries": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i, _i, _i, _vp, _vp, _vp, _vp,
                                    _vp]),
    "sb_route_workspace_bytes": (_i64, [_i, _i, _i, _i]),
    "sb_route_topk": (_i, [_vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i, _f, _vp, _vp, _vp, _vp]),
    "sb_route_topk_head_budgets": (_i, [_vp, _vp, _i, _i, _i, _i, _i, _i, _i, _vp, _i, _f, _vp, _vp, _vp, _vp]),
    "sb_route_topk_noalloc": (_i, [_vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i, _f, _vp, _vp, _vp]),
    "sb_sparse_attention": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _vp, _i, _vp, _vp, _vp, _i, _i, _i, _i,
                                 _vp, _vp, _vp]),
    "sb_route_pair_workspace_bytes": (_i64, [_i, _i, _i]),
    "sb_route_pair_blocks": (_i, [_vp, _i, _i, _i, _i, _i, _vp, _vp, _vp]),
    "sb_sparse_attention_pairs": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _vp, _i, _vp, _vp, _vp, _i, _i, _i,
                                       _i, _vp, _vp, _vp, _vp]),
    "sb_selftest_wait_timeout": (_i, [ctypes.c_longlong, _vp, _vp]),
    "sb_dense_rows_attention": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _vp, _vp, _vp]),
    "sb_tail_summaries8": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i, _i, _vp, _vp, _vp, _vp]),
    "sb_tail_merge": (_i, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _i, _vp, _i, _i, _i, _i, _i, _vp, _vp,
                           _vp]),
    "sb_headwise_permute": (_i, [_vp, _vp, _vp, _i, _i, _i, _i, _i, _i, _i, _vp]),
    "sb_fp8_quantize_rows": (_i, [_vp, _i, _i64, _i, _vp, _vp, _vp]),
    "sb_fp8_swiglu_quantize_rows": (_i, [_vp, _i, _i64, _i, _vp, _vp, _vp]),
    "sb_fp8_quantize_tensor": (_i, [_vp, _i, _i64, _vp, _vp, _vp, _vp]),
    "sb_fp8_swiglu": (_i, [_vp, _i, _i64, _i, _vp, _vp]),
    "sb_fp8_gemm": (_i, [_vp, _vp, _i, _vp, _vp, _i, _i64, _i, _i, _vp, _vp, _i, _vp]),
    "sb_fp8_gemm_qkv_rope": (_i, [_vp, _vp, _vp, _vp, _i64, _i, _i, _vp, _vp, _vp, _vp, _i, _vp, _vp, _i, ctypes.c_float,
                                  _vp, _vp, _vp, _i, _vp]),
    "sb_fp8_gemm_qkv_rope_peers": (_i, [_vp, _vp, _vp, _vp, _i64, _i, _i, _vp, _vp, _vp, _vp, _i, _vp, _vp, _i, _i,
                                        ctypes.c_float, _vp, _i, _vp]),
    "sb_ipc_alloc": (_i, [_i64, _vp]),
    "sb_ipc_free": (_i, [_vp]),
    "sb_ipc_handle": (_i, [_vp, _vp]),
    "sb_ipc_open": (_i, [_vp, _vp]),
    "sb_ipc_close": (_i, [_vp]),
    "sb_fp8_gemm_residual": (_i, [_vp, _vp, _i, _vp, _vp, _i, _i64, _i, _i, _vp, _vp, _vp, _vp, _i, _vp]),
    "sb_fp8_gelu_quantize_rows": (_i, [_vp, _i, _i64, _i, _vp, _vp, _vp]),
    "sb_fp8_quantize_segments": (_i, [_vp, _i64, _i, _i, _i64, _vp, _vp, _vp]),
    "sb_dit_norm_modulate_quantize": (_i, [_vp, _vp, _vp, _i64, _i, ctypes.c_float, _vp, _vp, _vp]),
    "sb_dit_qkv_norm_rope": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i, _i, _i, ctypes.c_float, _vp, _vp, _vp, _vp]),
    "sb_memcpy2d": (_i, [_vp, _i64, _vp, _i64, _i64, _i64, _vp]),
    "sb_reblock_metric": (_i, [_vp, _vp, _i, _i, _i, _i, _i, _vp, _i, ctypes.c_float, _vp, _vp]),
    "sb_reblock_transform": (_i, [_vp, _vp, _i, _i, _i, _i, _i, _vp, _vp, _vp]),
    "sb_reblock_plan": (_i64, [_vp, _i, _i, _vp, _i64]),
    "sb_reblock_plan_proxy": (_i, [_vp, _i, _i]),
    "sb_reblock_workspace_bytes": (_i64, [_vp, _i]),
    "sb_reblock_tree": (_i, [_vp, _i, _i, _i, _vp, _vp, _vp, _vp, _i64, _vp, _vp, _vp]),
    "sb_reblock_tree_frozen": (_i, [_vp, _i, _i, _i, _vp, _vp, _vp, _vp, _vp, _i64, _vp, _vp, _vp]),
    "sb_reblock_remainder": (_i, [_vp, _i, _i, _i, _vp, _i64, _vp, _vp]),
}


class SparkKernelError(RuntimeError):
    """A C-ABI call returned a negative status."""


def load(build_if_missing: bool = True) -> ctypes.CDLL:
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = _build.LIB_PATH
        if not path.exists() or _build.stale():
            if not build_if_missing:
                raise RuntimeError(f"spark_h3_b200 native library is missing or out of date: {path}")
            _build.build()
        lib = ctypes.CDLL(str(path))
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        _lib = lib
        return lib


def check(status: int, what: str) -> None:
    if status < 0:
        message = load().sb_last_error().decode(errors="replace")
        raise SparkKernelError(f"{what} failed ({status}): {message}")


def call(name: str, *args) -> int:
    status = getattr(load(), name)(*args)
    check(status, name)
    return status
