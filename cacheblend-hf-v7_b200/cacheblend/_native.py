"""ctypes binding of libcbk.so (the sm_100a kernels, C ABI in include/cbk.h).

The library is loaded when the package is imported; a missing library is an
ImportError, never a silent fallback.
"""
from __future__ import annotations

import ctypes
import os

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib", "libcbk.so")

CBK_OK = 0
CBK_ERR_INVALID = -1
CBK_ERR_UNSUPPORTED = -2
CBK_ERR_CUDA = -3
CBK_ERR_WORKSPACE = -4
CBK_BF16, CBK_F16 = 0, 1
CBK_ROPE_REF, CBK_ROPE_FP32 = 0, 1
CBK_ROPE_TABLE_BY_ROW = 16
CBK_STATUS_BAD_INDEX, CBK_STATUS_TIMEOUT, CBK_STATUS_COUNT = 1, 2, 4

_vp, _i32, _i64, _f32, _f64, _sz = (ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float,
                                    ctypes.c_double, ctypes.c_size_t)

# name -> (restype, argtypes); mirrors include/cbk.h
SIGNATURES = {
    "cbk_last_error": (ctypes.c_char_p, []),
    "cbk_abi_version": (_i32, []),
    "cbk_rope_table": (_i32, [_vp, _i32, _i64, _f32, _vp, _vp]),
    "cbk_assemble_kv": (_i32, [_vp, _vp, _i32, _i32, _i64, _i32, _i32, _i32, _vp, _i64, _vp, _i32,
                               _vp, _vp, _i64, _vp, _vp]),
    "cbk_rope_rows": (_i32, [_vp, _vp, _i64, _i32, _i32, _i32, _vp, _i64, _vp, _i32, _vp, _vp]),
    "cbk_rope_scatter": (_i32, [_vp, _i64, _vp, _i64, _vp, _i64, _i32, _vp, _i64, _i64, _i32, _i32,
                                _i32, _i32, _vp, _i64, _i32, _vp, _vp, _vp, _vp, _vp]),
    "cbk_kv_deviation": (_i32, [_vp, _i64, _vp, _vp, _i32, _i64, _i64, _i32, _vp, _vp]),
    "cbk_topk_count": (_i64, [_i64, _f64]),
    "cbk_topk_select": (_i32, [_vp, _i64, _i64, _i32, _vp, _vp, _vp]),
    "cbk_hkvd_workspace_bytes": (_sz, [_i64]),
    "cbk_hkvd_select": (_i32, [_vp, _i64, _vp, _vp, _i32, _i64, _i64, _i32, _i64, _i32, _vp, _vp,
                               _sz, _vp, _vp]),
    "cbk_hkvd_noalloc_max_tokens": (_i64, []),
    "cbk_hkvd_select_noalloc": (_i32, [_vp, _i64, _vp, _vp, _i32, _i64, _i64, _i32, _i64, _i32, _vp,
                                       _vp, _vp]),
    "cbk_partial_attn_workspace_bytes": (_sz, [_i64, _i64, _i32, _i32, _i32]),
    "cbk_partial_attn": (_i32, [_vp, _vp, _vp, _vp, _i64, _i64, _i32, _i32, _i32, _f32, _i32, _vp,
                                _vp, _sz, _i32, _vp, _vp]),
    "cbk_add_rmsnorm": (_i32, [_vp, _i64, _i64, _vp, _vp, _i64, _vp, _i64, _vp, _f32, _i64, _i32, _i32,
                               _vp, _i64, _vp, _vp]),
    "cbk_silu_mul": (_i32, [_vp, _i64, _vp, _i64, _i64, _i32, _i32, _vp, _i64, _vp]),
    "cbk_scatter_rows": (_i32, [_vp, _i64, _vp, _i64, _vp, _i64, _i64, _i64, _vp]),
    "cbk_gemv": (_i32, [_vp, _i64, _vp, _vp, _vp, _i64, _i32, _i32, _vp, _vp]),
    "cbk_decode_attn_workspace_bytes": (_sz, [_i64, _i32, _i32, _i32]),
    "cbk_decode_attn": (_i32, [_vp, _vp, _vp, _i64, _vp, _i64, _i32, _i32, _i32, _f32, _i32, _vp, _vp, _sz,
                               _vp, _vp]),
}


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"libcbk.so not found at {LIB_PATH}; build it with `python cacheblend-hf-v7_b200/build.py` "
            "(needs nvcc).  There is no CPU fallback.")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if lib.cbk_abi_version() != 1:
        raise ImportError("libcbk.so ABI version mismatch")
    return lib


LIB = _load()


def last_error() -> str:
    msg = LIB.cbk_last_error()
    return msg.decode(errors="replace") if msg else ""


def check(rc: int, fn: str) -> None:
    """Map a C-ABI return code to the exception type the reference raises."""
    if rc == CBK_OK:
        return
    msg = f"{fn}: {last_error()}"
    if rc == CBK_ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    if rc in (CBK_ERR_INVALID, CBK_ERR_WORKSPACE):
        raise ValueError(msg)
    raise RuntimeError(msg)
