"""HKVD selection (API of cacheblend-hf-v7 ``hkvd.py``) on the sm_100a kernels.

``kv_deviation`` and ``select_top_k`` keep the reference's signatures, shapes,
dtypes and exceptions; the arithmetic runs in ``deviation_kernel`` (fp32, fixed
reduction order) and ``topk_kernel`` (radix select, ascending indices, ties at
the k-th value taken lowest index first).
"""
from __future__ import annotations

import torch

from cacheblend import ops


class _PlainRows:
    """Minimal chunk table over one (S, F) tensor, for the plain API."""

    def __init__(self, rows: torch.Tensor):
        dev = rows.device
        self.S = rows.shape[0]
        self.n_chunks = 1
        self._rows = rows
        host = torch.tensor([[rows.data_ptr(), rows.data_ptr()]], dtype=torch.int64)
        self.srcs = host.to(dev)
        self.starts = torch.tensor([0, self.S], dtype=torch.int64, device=dev)
        self.layers = [0]

    def layer_ptr(self, layer: int) -> int:
        return self.srcs.data_ptr()


def kv_deviation(K_new: torch.Tensor, K_old: torch.Tensor) -> torch.Tensor:
    """Per-token squared-L2 deviation, fp32 (S,) -- reference hkvd.py:23-55.

    Accepts (1, S, F) or (S, F).  Raises ValueError on a shape mismatch or other
    ndim and NotImplementedError for batch > 1, like the reference."""
    if K_new.shape != K_old.shape:
        raise ValueError(f"shape mismatch: K_new={K_new.shape}, K_old={K_old.shape}")
    if K_new.ndim == 3:
        if K_new.shape[0] != 1:
            raise NotImplementedError("kv_deviation: batch>1 not supported in Phase 3")
        a, b = K_new[0], K_old[0]
    elif K_new.ndim == 2:
        a, b = K_new, K_old
    else:
        raise ValueError(f"unsupported ndim: {K_new.ndim}")
    ops.require_cuda(a, b)
    ops.dtype_code(a.dtype)
    if b.dtype != a.dtype:
        b = b.to(a.dtype)
    a = a if (a.stride(-1) == 1 and a.data_ptr() % 16 == 0) else a.contiguous()
    b = b.contiguous()
    if b.data_ptr() % 16:
        b = b.clone()
    return ops.kv_deviation_rows(a, _PlainRows(b), 0)


def select_top_k(deviations: torch.Tensor, ratio: float) -> torch.Tensor:
    """Indices of the int(S * ratio) (>= 1, <= S) largest deviations, ascending,
    int64 on the deviations' device -- reference hkvd.py:58-77."""
    S = deviations.shape[0]
    k = max(1, min(S, int(S * ratio)))
    return ops.topk_select(deviations, k, force_last=False)
