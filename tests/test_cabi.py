"""The C-ABI library loads, exports every symbol include/cbk.h declares, and
rejects bad arguments with error codes before touching the GPU.  CPU only."""
import ctypes
import os
import re

import pytest

from conftest import ROOT


def _declared():
    src = open(os.path.join(ROOT, "include", "cbk.h")).read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?[\w\s\*]+?\b(cbk_\w+)\s*\(", src, re.M)))


def test_header_declares_entry_points():
    names = _declared()
    for n in ("cbk_assemble_kv", "cbk_rope_scatter", "cbk_kv_deviation", "cbk_topk_select",
              "cbk_hkvd_select", "cbk_partial_attn", "cbk_last_error", "cbk_rope_table"):
        assert n in names


def test_library_exports_every_declared_symbol():
    from cacheblend import _native
    lib = ctypes.CDLL(_native.LIB_PATH)
    missing = [n for n in _declared() if not hasattr(lib, n)]
    assert not missing, missing
    assert set(_native.SIGNATURES) == set(_declared())


def test_abi_version_and_pure_helpers():
    from cacheblend import _native as N
    assert N.LIB.cbk_abi_version() == 1
    for S in (1, 7, 544, 6208, 131328):
        for r in (1e-9, 0.15, 0.5, 1.0, 2.0):
            assert N.LIB.cbk_topk_count(S, r) == max(1, min(S, int(S * r)))
    assert N.LIB.cbk_hkvd_workspace_bytes(6208) >= 6208 * 4
    assert N.LIB.cbk_hkvd_workspace_bytes(6208) % 256 == 0
    # decode attention: per-split partials sized for the split maximum, whatever the cache length
    dec = N.LIB.cbk_decode_attn_workspace_bytes(6240, 32, 8, 128)
    assert dec >= 8 * 64 * 4 * 128 * 4 and dec == N.LIB.cbk_decode_attn_workspace_bytes(131328, 32, 8, 128)
    assert N.LIB.cbk_decode_attn_workspace_bytes(0, 32, 8, 128) == 0
    assert N.LIB.cbk_decode_attn_workspace_bytes(100, 32, 3, 128) == 0


@pytest.mark.parametrize("call,code", [
    ("cbk_topk_select(None, 10, 0, 0, None, None, None)", -1),
    ("cbk_topk_select(1024, 10, 11, 0, 2048, None, None)", -1),
    ("cbk_partial_attn(16, 16, 16, 16, 4, 8, 4, 2, 96, 0.1, 0, 16, 16, 1 << 30, 0, None, None)", -2),
    ("cbk_partial_attn(16, 16, 16, 16, 4, 8, 12, 4, 128, 0.1, 0, 16, 16, 1 << 30, 0, None, None)", -2),
    ("cbk_partial_attn(16, 16, 16, 16, 4, 8, 4, 2, 128, 0.1, 7, 16, 16, 1 << 30, 0, None, None)", -2),
    ("cbk_partial_attn(16, 16, 16, 16, 4, 8, 5, 2, 128, 0.1, 0, 16, 16, 1 << 30, 0, None, None)", -1),
    ("cbk_partial_attn(16, 16, 16, 16, 9, 8, 4, 2, 128, 0.1, 0, 16, 16, 1 << 30, 0, None, None)", -1),
    ("cbk_partial_attn(16, 16, 16, 16, 4, 8, 4, 2, 128, 0.1, 0, 16, None, 1 << 30, 0, None, None)", -1),
    ("cbk_partial_attn(16, 16, 16, 16, 4, 8, 4, 2, 128, 0.1, 0, 16, 16, 64, 0, None, None)", -4),
    ("cbk_assemble_kv(None, None, 1, 1, 8, 2, 64, 0, None, 8, None, 0, None, None, 0, None, None)", -1),
    ("cbk_assemble_kv(16, 16, 1, 1, 8, 2, 40, 0, 16, 8, None, 0, 16, 16, 1024, None, None)", -2),
    ("cbk_rope_scatter(16, 8, 16, 8, 16, 8, 0, 16, 1, 8, 3, 2, 64, 0, 16, 8, 0, 16, 16, 16, None, None)", -1),
    ("cbk_kv_deviation(16, 12, 16, 16, 1, 8, 12, 0, 16, None)", -1),
    ("cbk_hkvd_select(16, 8, 16, 16, 1, 8, 8, 0, 2, 1, 16, 16, 4, None, None)", -4),
    ("cbk_rope_rows(16, 16, 4, 2, 64, 1, 16, 8, 16, 5, None, None)", -1),
    # add_rmsnorm(x, xs, x_rows, rows, delta, ds, sum, ss, w, eps, n_rows, cols, dtype, out, os, status, stream)
    ("cbk_add_rmsnorm(16, 64, 4, None, None, 0, None, 0, 16, 1e-5, 4, 64, 3, 16, 64, None, None)", -2),
    ("cbk_add_rmsnorm(16, 64, 4, None, None, 0, None, 0, 16, 1e-5, 4, 60, 0, 16, 64, None, None)", -1),
    ("cbk_add_rmsnorm(16, 9000, 4, None, None, 0, None, 0, 16, 1e-5, 4, 8200, 0, 16, 9000, None, None)", -1),
    ("cbk_add_rmsnorm(None, 64, 4, None, None, 0, None, 0, 16, 1e-5, 4, 64, 0, 16, 64, None, None)", -1),
    ("cbk_add_rmsnorm(16, 32, 4, None, None, 0, None, 0, 16, 1e-5, 4, 64, 0, 16, 64, None, None)", -1),
    ("cbk_add_rmsnorm(18, 64, 4, None, None, 0, None, 0, 16, 1e-5, 4, 64, 0, 16, 64, None, None)", -1),
    ("cbk_add_rmsnorm(16, 64, 4, None, None, 0, None, 0, 16, 1e-5, 5, 64, 0, 16, 64, None, None)", -1),
    ("cbk_add_rmsnorm(16, 64, 4, None, None, 0, None, 0, 16, 1e-5, 0, 64, 0, 16, 64, None, None)", 0),
    ("cbk_silu_mul(16, 64, 16, 64, 4, 64, 2, 16, 64, None)", -2),
    ("cbk_silu_mul(16, 64, 16, 64, 4, 12, 0, 16, 64, None)", -1),
    ("cbk_silu_mul(16, 64, None, 64, 4, 64, 0, 16, 64, None)", -1),
    ("cbk_silu_mul(16, 64, 16, 60, 4, 64, 0, 16, 64, None)", -1),
    ("cbk_silu_mul(16, 64, 16, 64, 0, 64, 0, 16, 64, None)", 0),
    # scatter_rows(src, src_stride, idx, k, dst, dst_stride, S, row_bytes, stream)
    ("cbk_gemv(16, 64, 16, None, None, 4, 64, 2, 16, None)", -2),
    ("cbk_gemv(16, 64, 16, None, None, 4, 12, 0, 16, None)", -1),
    ("cbk_gemv(16, 64, 16, None, None, 4, 64, 0, None, None)", -1),
    ("cbk_gemv(16, 64, None, 16, None, 4, 64, 0, 16, None)", -1),
    ("cbk_gemv(24, 64, 16, None, None, 4, 64, 0, 16, None)", -1),
    ("cbk_gemv(16, 60, 16, None, None, 4, 64, 0, 16, None)", -1),
    ("cbk_gemv(16, 32768, 16, None, None, 4, 32768, 0, 16, None)", -1),
    ("cbk_gemv(16, 64, 16, None, None, 0, 64, 0, 16, None)", 0),
    ("cbk_decode_attn(16, 16, 16, 1024, 16, 100, 32, 8, 128, 0.1, 2, 16, 16, 1 << 20, None, None)", -2),
    ("cbk_decode_attn(16, 16, 16, 1024, 16, 100, 32, 8, 96, 0.1, 0, 16, 16, 1 << 20, None, None)", -2),
    ("cbk_decode_attn(16, 16, 16, 1024, 16, 100, 32, 2, 128, 0.1, 0, 16, 16, 1 << 20, None, None)", -2),
    ("cbk_decode_attn(16, 16, 16, 1000, 16, 100, 32, 8, 128, 0.1, 0, 16, 16, 1 << 20, None, None)", -1),
    ("cbk_decode_attn(16, 16, 16, 1024, None, 100, 32, 8, 128, 0.1, 0, 16, 16, 1 << 20, None, None)", -1),
    ("cbk_decode_attn(16, 24, 16, 1024, 16, 100, 32, 8, 128, 0.1, 0, 16, 16, 1 << 20, None, None)", -1),
    ("cbk_decode_attn(16, 16, 16, 1024, 16, 100, 32, 8, 128, 0.1, 0, 16, 16, 64, None, None)", -4),
    ("cbk_scatter_rows(16, 64, 16, 2, None, 64, 4, 64, None)", -1),
    ("cbk_scatter_rows(16, 64, 16, 5, 16, 64, 4, 64, None)", -1),
    ("cbk_scatter_rows(16, 64, 16, 2, 16, 64, 4, 60, None)", -1),
    ("cbk_scatter_rows(16, 64, 16, 2, 24, 64, 4, 64, None)", -1),
    ("cbk_scatter_rows(16, 32, 16, 2, 16, 64, 4, 64, None)", -1),
    ("cbk_scatter_rows(16, 64, 16, 0, 16, 64, 0, 64, None)", 0),
])
def test_validation_errors_before_any_launch(call, code):
    from cacheblend import _native as N
    rc = eval("N.LIB." + call)
    assert rc == code, (call, rc, N.last_error())
    assert N.last_error()


def test_error_codes_map_to_reference_exceptions():
    from cacheblend import _native as N
    with pytest.raises(ValueError):
        N.check(N.CBK_ERR_INVALID, "x")
    with pytest.raises(NotImplementedError):
        N.check(N.CBK_ERR_UNSUPPORTED, "x")
    with pytest.raises(RuntimeError):
        N.check(N.CBK_ERR_CUDA, "x")
