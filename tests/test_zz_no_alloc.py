"""The no-allocation HKVD entry point (cbk_hkvd_select_noalloc), called through
the C ABI, must select exactly what the allocating entry point (cbk_hkvd_select,
caller workspace) selects.

It exists for callers that cannot allocate device memory when they pick the
tokens to recompute: an engine that has already reserved the HBM for its own
pools, or a latency-critical step where cudaMalloc would synchronise the
device.  Its deviation scores live in a fixed library-owned device array that
all calls share, so two calls in a row are checked (the second on a shorter
sequence, which must not see the first call's leftovers), and a sequence longer
than the array is rejected with a clear error.  Indices are integer results:
compared bit for bit, the bar every HKVD test here uses.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _case(lengths, feat, seed):
    from cacheblend import ops
    g = torch.Generator().manual_seed(seed)
    entries = [{"K": [(torch.randn((1, n, feat), generator=g) * 2).to(torch.bfloat16).to(DEV)],
                "V": [torch.randn((1, n, feat), generator=g).to(torch.bfloat16).to(DEV)]}
               for n in lengths]
    S = sum(lengths)
    old = torch.cat([e["K"][0][0] for e in entries]).float().cpu()
    mask = (torch.rand((S, 1), generator=g) < 0.2).float()
    new = (old + torch.randn((S, feat), generator=g) * 0.05 * mask).to(torch.bfloat16).to(DEV)
    table = ops.ChunkTable(entries, [0], DEV)
    return new, table, S


def _select_allocating(N, new, table, S, feat, k):
    ws_bytes = int(N.LIB.cbk_hkvd_workspace_bytes(S))
    ws = torch.empty((ws_bytes // 4,), dtype=torch.float32, device=DEV)
    idx = torch.empty((k,), dtype=torch.int64, device=DEV)
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    stream = ctypes.c_void_p(torch.cuda.current_stream(DEV).cuda_stream)
    rc = N.LIB.cbk_hkvd_select(ctypes.c_void_p(new.data_ptr()), new.stride(0),
                               ctypes.c_void_p(table.layer_ptr(0)), ctypes.c_void_p(table.starts.data_ptr()),
                               table.n_chunks, S, feat, N.CBK_BF16, k, 1, ctypes.c_void_p(idx.data_ptr()),
                               ctypes.c_void_p(ws.data_ptr()), ws_bytes, ctypes.c_void_p(st.data_ptr()),
                               stream)
    assert rc == 0, N.last_error()
    return idx, st


def _select_noalloc(N, new, table, S, feat, k):
    idx = torch.empty((k,), dtype=torch.int64, device=DEV)
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    stream = ctypes.c_void_p(torch.cuda.current_stream(DEV).cuda_stream)
    rc = N.LIB.cbk_hkvd_select_noalloc(ctypes.c_void_p(new.data_ptr()), new.stride(0),
                                       ctypes.c_void_p(table.layer_ptr(0)),
                                       ctypes.c_void_p(table.starts.data_ptr()), table.n_chunks, S, feat,
                                       N.CBK_BF16, k, 1, ctypes.c_void_p(idx.data_ptr()),
                                       ctypes.c_void_p(st.data_ptr()), stream)
    assert rc == 0, N.last_error()
    return idx, st


@pytest.mark.parametrize("cases", [
    [([1024] * 6 + [64], 1024, 1), ([128] * 4 + [32], 256, 2)],          # 2nd call: shorter S
    # above the top-K kernel's shared-memory key cache (40960 keys: the scores are
    # read back from the scratch array itself), then the scratch array's full length
    [([20481, 20481], 128, 4), ([65536] * 4, 128, 5)],
])
def test_noalloc_hkvd_matches_allocating_entry_point_twice(cases):
    from cacheblend import _native as N
    for lengths, feat, seed in cases:
        new, table, S = _case(lengths, feat, seed)
        k = int(N.LIB.cbk_topk_count(S, 0.15))
        a, sa = _select_allocating(N, new, table, S, feat, k)
        b, sb = _select_noalloc(N, new, table, S, feat, k)
        torch.cuda.synchronize()
        assert int(sa.item()) == 0 and int(sb.item()) == 0
        np.testing.assert_array_equal(b.cpu().numpy(), a.cpu().numpy())
        assert int(b[-1]) == S - 1
    if sum(cases[-1][0]) == 4 * 65536:
        assert sum(cases[-1][0]) == int(N.LIB.cbk_hkvd_noalloc_max_tokens())


def test_noalloc_rejects_sequences_beyond_its_scratch():
    from cacheblend import _native as N
    new, table, _ = _case([64, 64], 128, 3)
    limit = int(N.LIB.cbk_hkvd_noalloc_max_tokens())
    assert limit >= 131328                     # covers a 128K-token blended prompt
    idx = torch.empty((8,), dtype=torch.int64, device=DEV)
    rc = N.LIB.cbk_hkvd_select_noalloc(ctypes.c_void_p(new.data_ptr()), new.stride(0),
                                       ctypes.c_void_p(table.layer_ptr(0)),
                                       ctypes.c_void_p(table.starts.data_ptr()), table.n_chunks,
                                       limit + 1, 128, N.CBK_BF16, 8, 1, ctypes.c_void_p(idx.data_ptr()),
                                       None, ctypes.c_void_p(torch.cuda.current_stream(DEV).cuda_stream))
    assert rc == N.CBK_ERR_INVALID
    assert "exceeds the fixed scratch" in N.last_error()
