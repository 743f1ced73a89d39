"""torch-facing wrappers of the libcbk kernels.

Each wrapper validates devices, dtypes, shapes and contiguity, passes raw
device pointers plus the current CUDA stream to the C ABI, and maps return
codes to Python exceptions.  Nothing here runs on the CPU: a non-CUDA tensor is
an error.
"""
from __future__ import annotations

import ctypes
from typing import Sequence

import numpy as np

import torch

from cacheblend import _native as N
from cacheblend._timing import TIMES

_DT = {torch.bfloat16: N.CBK_BF16, torch.float16: N.CBK_F16}
ROPE_MODES = {"ref": N.CBK_ROPE_REF, "fp32": N.CBK_ROPE_FP32}


def _vp(x) -> ctypes.c_void_p:
    if x is None:
        return ctypes.c_void_p(0)
    return ctypes.c_void_p(x.data_ptr() if isinstance(x, torch.Tensor) else int(x))


def _stream(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def dtype_code(dt: torch.dtype) -> int:
    if dt not in _DT:
        raise NotImplementedError(f"libcbk kernels support bfloat16/float16 tensors, got {dt}")
    return _DT[dt]


def require_cuda(*ts: torch.Tensor) -> torch.device:
    dev = None
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError("cacheblend kernels need CUDA tensors (no CPU path); got a "
                               f"{t.device} tensor")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"tensors on different devices: {dev} and {t.device}")
    return dev


def _rows(t: torch.Tensor, name: str) -> torch.Tensor:
    """Flatten to 2-D rows with unit inner stride and 16-byte aligned rows."""
    t2 = t.reshape(-1, t.shape[-1])
    if t2.stride(-1) != 1 or t2.stride(0) % 8 or t2.data_ptr() % 16:
        t2 = t2.contiguous()
    return t2


# ---------------------------------------------------------------------------
# RoPE
# ---------------------------------------------------------------------------
def rope_table(inv_freq: torch.Tensor, n_pos: int, scaling: float = 1.0) -> torch.Tensor:
    """(n_pos, D/2, 2) fp32 cos/sin table for positions 0..n_pos-1."""
    dev = require_cuda(inv_freq)
    inv = inv_freq.to(device=dev, dtype=torch.float32).contiguous()
    half = inv.numel()
    table = torch.empty((int(n_pos), half, 2), dtype=torch.float32, device=dev)
    with TIMES.span("rope_table", dev):
        N.check(N.LIB.cbk_rope_table(_vp(inv), half, int(n_pos), float(scaling), _vp(table), _stream(dev)),
              "cbk_rope_table")
    return table


def rope_rows(x: torch.Tensor, positions: torch.Tensor, table: torch.Tensor, head_dim: int,
              mode: str = "ref", out: torch.Tensor | None = None, status=None) -> torch.Tensor:
    """out[r] = RoPE(x[r], positions[r]) for rows of n_heads*head_dim elements."""
    dev = require_cuda(x, positions, table)
    xr = _rows(x, "x")
    pos = positions.reshape(-1).to(device=dev, dtype=torch.int64).contiguous()
    if pos.numel() != xr.shape[0]:
        raise ValueError(f"positions ({pos.numel()}) must match rows ({xr.shape[0]})")
    if out is None:
        out = torch.empty_like(xr)
    n_heads = xr.shape[1] // head_dim
    if n_heads * head_dim != xr.shape[1]:
        raise ValueError(f"row width {xr.shape[1]} is not a multiple of head_dim {head_dim}")
    with TIMES.span("rope_rows", dev):
        N.check(N.LIB.cbk_rope_rows(_vp(xr), _vp(out), xr.shape[0], n_heads, head_dim,
                                  dtype_code(x.dtype), _vp(table), table.shape[0], _vp(pos),
                                  ROPE_MODES[mode], _vp(status), _stream(dev)), "cbk_rope_rows")
    return out.view(x.shape)


# ---------------------------------------------------------------------------
# chunk tables
# ---------------------------------------------------------------------------
class ChunkTable:
    """Device descriptor table of chunk tensors: [layer][chunk] -> (K ptr, V ptr),
    plus the chunk start offsets (n_chunks + 1) in the fused sequence.

    Holds references to the chunk tensors so they outlive the kernels."""

    def __init__(self, entries: Sequence[dict], layers: Sequence[int], device: torch.device):
        self.n_chunks = len(entries)
        self.layers = list(layers)
        lens = []
        self._keep = []
        host = torch.empty((len(self.layers), self.n_chunks, 2), dtype=torch.int64, pin_memory=True)
        hv = host.numpy()
        kv_dim = None
        slabs = [e.get("_slab") for e in entries]
        if self.n_chunks and all(sl is not None for sl in slabs) and \
                len({(sl[0], sl[3], sl[4], sl[5]) for sl in slabs}) == 1:
            # chunks of one KVArena: the table follows from the slab offsets
            pool, _, _, row_elems, n_layers, kv_dim = slabs[0]
            t0 = entries[0]["K"][self.layers[0]]
            if t0.device != device:
                raise RuntimeError(f"chunk tensor on {t0.device}, model on {device}")
            esz = t0.element_size()
            first = np.array([sl[1] for sl in slabs], dtype=np.int64)
            lens_a = np.array([sl[2] for sl in slabs], dtype=np.int64)
            lay = np.array(self.layers, dtype=np.int64)
            if lay.min() < 0 or lay.max() >= n_layers:
                raise ValueError("chunk table layer out of range of the arena")
            kptr = pool + (first * row_elems)[None, :] * esz + lay[:, None] * (2 * lens_a * kv_dim * esz)[None, :]
            hv[:, :, 0] = kptr
            hv[:, :, 1] = kptr + (lens_a * kv_dim * esz)[None, :]
            lens = lens_a.tolist()
            self._keep = [e["K"][self.layers[0]] for e in entries]   # views keep the pool alive
            self._finish(host, lens, kv_dim, t0.dtype, device)
            return
        for c, e in enumerate(entries):
            for li, l in enumerate(self.layers):
                k = _chunk_rows(e["K"][l], device)
                v = _chunk_rows(e["V"][l], device)
                if k.shape != v.shape:
                    raise ValueError("chunk K and V shapes differ")
                if kv_dim is None:
                    kv_dim = k.shape[1]
                if k.shape[1] != kv_dim:
                    raise ValueError("chunk tensors have different widths")
                self._keep += [k, v]
                hv[li, c, 0] = k.data_ptr()
                hv[li, c, 1] = v.data_ptr()
                if li == 0:
                    lens.append(k.shape[0])
                elif k.shape[0] != lens[c]:
                    raise ValueError("chunk length differs across layers")
        self._finish(host, lens, kv_dim, self._keep[0].dtype, device)

    def _finish(self, host, lens, kv_dim, dtype, device):
        starts = [0]
        for n in lens:
            starts.append(starts[-1] + n)
        hs = torch.tensor(starts, dtype=torch.int64).pin_memory()
        self.kv_dim = kv_dim
        self.S = starts[-1]
        self.lengths = lens
        self.srcs = host.to(device, non_blocking=True)
        self.starts = hs.to(device, non_blocking=True)
        self.dtype = dtype

    def refresh(self, entries: Sequence[dict]) -> None:
        """Point the same device table at other chunks of the same lengths
        (a captured graph reads it in place); ordered on the current stream."""
        new = ChunkTable(entries, self.layers, self.srcs.device)
        if new.lengths != self.lengths or new.kv_dim != self.kv_dim or new.dtype != self.dtype:
            raise ValueError("ChunkTable.refresh: chunk lengths / width / dtype differ from the table's")
        self.srcs.copy_(new.srcs, non_blocking=True)
        self._keep = new._keep

    def layer_ptr(self, layer: int) -> int:
        """Device address of the srcs row of one layer (n_chunks entries)."""
        li = self.layers.index(layer)
        return self.srcs.data_ptr() + li * self.n_chunks * 16


def chunk_signature(entries: Sequence[dict], layers: Sequence[int]) -> tuple:
    """Device addresses of the store entries' K/V tensors of `layers` (for
    KVArena entries, their slab): equal signatures mean a ChunkTable built from
    either set of entries holds the same pointers.  (A table keeps its tensors
    alive, so a stored tensor that replaced one of them cannot have its address.)"""
    sig = []
    for e in entries:
        slab = e.get("_slab")
        if slab is not None:
            sig.append(slab)
        else:
            K, V = e["K"], e["V"]
            sig.append(tuple(K[l].data_ptr() for l in layers) + tuple(V[l].data_ptr() for l in layers))
    return tuple(sig)


def _chunk_rows(t: torch.Tensor, device) -> torch.Tensor:
    if t.device != device:
        raise RuntimeError(f"chunk tensor on {t.device}, model on {device}")
    t2 = t.reshape(-1, t.shape[-1])
    if not t2.is_contiguous() or t2.data_ptr() % 16:
        t2 = t2.contiguous()
    return t2


# ---------------------------------------------------------------------------
# (a)+(b) assemble, (b)+(d) fresh-row scatter
# ---------------------------------------------------------------------------
def assemble_kv(table: ChunkTable, layer_lo: int, layer_hi: int, n_kv_heads: int, head_dim: int,
                rope: torch.Tensor, k_out: torch.Tensor, v_out: torch.Tensor, mode: str = "ref",
                positions: torch.Tensor | None = None, status=None) -> None:
    """Fill k_out[l], v_out[l] (l in [layer_lo, layer_hi)) of [L][S][kv_dim]
    buffers from the chunk tensors, K rotated to its fused positions."""
    dev = require_cuda(k_out, v_out, rope)
    n_layers = layer_hi - layer_lo
    if n_layers <= 0:
        return
    li0 = table.layers.index(layer_lo)
    if table.layers[li0:li0 + n_layers] != list(range(layer_lo, layer_hi)):
        raise ValueError("chunk table does not hold the requested consecutive layers")
    srcs = table.srcs.data_ptr() + li0 * table.n_chunks * 16
    lstride = k_out.stride(0)
    kb = k_out.data_ptr() + layer_lo * lstride * k_out.element_size()
    vb = v_out.data_ptr() + layer_lo * lstride * v_out.element_size()
    with TIMES.span("assemble_kv", dev):
        N.check(N.LIB.cbk_assemble_kv(_vp(srcs), _vp(table.starts), table.n_chunks, n_layers, table.S,
                                    n_kv_heads, head_dim, dtype_code(k_out.dtype), _vp(rope),
                                    rope.shape[0], _vp(positions), ROPE_MODES[mode], _vp(kb), _vp(vb),
                                    lstride, _vp(status), _stream(dev)), "cbk_assemble_kv")


def rope_scatter(q_src: torch.Tensor, k_src: torch.Tensor, v_src: torch.Tensor, idx: torch.Tensor,
                 gather: bool, S: int, n_q_heads: int, n_kv_heads: int, head_dim: int,
                 rope: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                 q_out: torch.Tensor | None = None, mode: str = "ref", status=None,
                 table_by_row: bool = False) -> torch.Tensor:
    """RoPE of fresh Q (-> q_out, [n_sel][Hq*D]) and K at positions idx; K and V
    rows written into the fused cache of one layer at rows idx.  With
    ``table_by_row`` row j of ``rope`` holds the cos/sin of position idx[j]
    (``rope.index_select(0, idx)``, made once per selection)."""
    dev = require_cuda(q_src, k_src, v_src, idx, rope, k_cache, v_cache)
    q2, k2, v2 = _rows(q_src, "q"), _rows(k_src, "k"), _rows(v_src, "v")
    n_sel = idx.numel()
    if q_out is None:
        q_out = torch.empty((n_sel, n_q_heads * head_dim), dtype=q_src.dtype, device=dev)
    with TIMES.span("rope_scatter", dev):
        N.check(N.LIB.cbk_rope_scatter(_vp(q2), q2.stride(0), _vp(k2), k2.stride(0), _vp(v2), v2.stride(0),
                                     int(bool(gather)), _vp(idx), n_sel, int(S), n_q_heads, n_kv_heads,
                                     head_dim, dtype_code(q_src.dtype), _vp(rope), rope.shape[0],
                                     ROPE_MODES[mode] | (N.CBK_ROPE_TABLE_BY_ROW if table_by_row else 0),
                                     _vp(q_out), _vp(k_cache), _vp(v_cache),
                                     _vp(status), _stream(dev)), "cbk_rope_scatter")
    return q_out


# ---------------------------------------------------------------------------
# (c) HKVD
# ---------------------------------------------------------------------------
def kv_deviation_rows(k_new: torch.Tensor, table: ChunkTable, layer: int) -> torch.Tensor:
    dev = require_cuda(k_new)
    kn = _rows(k_new, "K_new")
    out = torch.empty((table.S,), dtype=torch.float32, device=dev)
    with TIMES.span("kv_deviation", dev):
        N.check(N.LIB.cbk_kv_deviation(_vp(kn), kn.stride(0), _vp(table.layer_ptr(layer)),
                                     _vp(table.starts), table.n_chunks, table.S, kn.shape[1],
                                     dtype_code(k_new.dtype), _vp(out), _stream(dev)),
              "cbk_kv_deviation")
    return out


def topk_count(S: int, ratio: float) -> int:
    return int(N.LIB.cbk_topk_count(int(S), float(ratio)))


def topk_select(dev_scores: torch.Tensor, k: int, force_last: bool = False, status=None) -> torch.Tensor:
    dev = require_cuda(dev_scores)
    if dev_scores.dtype != torch.float32:
        dev_scores = dev_scores.float()
    d = dev_scores.contiguous()
    idx = torch.empty((int(k),), dtype=torch.int64, device=dev)
    with TIMES.span("topk_select", dev):
        N.check(N.LIB.cbk_topk_select(_vp(d), d.numel(), int(k), int(bool(force_last)), _vp(idx),
                                    _vp(status), _stream(dev)), "cbk_topk_select")
    return idx


def hkvd_select(k_new: torch.Tensor, table: ChunkTable, layer: int, k: int, force_last: bool = True,
                workspace: torch.Tensor | None = None, status=None):
    """Deviation of fresh K against the cached chunk K of `layer`, then top-K.
    Returns (indices, deviations) -- deviations live in the workspace."""
    dev = require_cuda(k_new)
    kn = _rows(k_new, "K_new")
    S = table.S
    need = int(N.LIB.cbk_hkvd_workspace_bytes(S))
    if workspace is None or workspace.numel() * workspace.element_size() < need:
        workspace = torch.empty((need // 4,), dtype=torch.float32, device=dev)
    idx = torch.empty((int(k),), dtype=torch.int64, device=dev)
    with TIMES.span("hkvd_select", dev, 2):
        N.check(N.LIB.cbk_hkvd_select(_vp(kn), kn.stride(0), _vp(table.layer_ptr(layer)),
                                    _vp(table.starts), table.n_chunks, S, kn.shape[1],
                                    dtype_code(k_new.dtype), int(k), int(bool(force_last)), _vp(idx),
                                    _vp(workspace), need, _vp(status), _stream(dev)),
              "cbk_hkvd_select")
    return idx, workspace.view(torch.float32)[:S]


# ---------------------------------------------------------------------------
# (e) partial attention
# ---------------------------------------------------------------------------
def attn_workspace(n_sel: int, S: int, n_q_heads: int, n_kv_heads: int, head_dim: int,
                   device) -> torch.Tensor:
    """Workspace for partial_attn (work plan + split partial results)."""
    nbytes = int(N.LIB.cbk_partial_attn_workspace_bytes(int(n_sel), int(S), n_q_heads, n_kv_heads, head_dim))
    if nbytes == 0:
        N.check(N.CBK_ERR_INVALID, "cbk_partial_attn_workspace_bytes")
    return torch.empty((nbytes,), dtype=torch.uint8, device=device)


def partial_attn(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, pos: torch.Tensor,
                 n_q_heads: int, n_kv_heads: int, head_dim: int, scale: float,
                 out: torch.Tensor | None = None, status=None, workspace: torch.Tensor | None = None,
                 reuse_plan: bool = False, timer_tag: str = "") -> torch.Tensor:
    """softmax(scale q k^T, keys <= pos) v for selected rows.

    q: [n_sel][Hq*D] (rotated); k_cache/v_cache: [S][Hkv*D]; pos: int64 [n_sel]
    ascending.  Returns [n_sel][Hq*D].  ``workspace`` (from attn_workspace) may
    be shared by calls with the same pos; ``reuse_plan`` skips re-planning."""
    dev = require_cuda(q, k_cache, v_cache, pos)
    n_sel = pos.numel()
    S = k_cache.shape[0]
    for t, name in ((q, "q"), (k_cache, "k_cache"), (v_cache, "v_cache")):
        if not t.is_contiguous():
            raise ValueError(f"partial_attn: {name} must be contiguous")
    if out is None:
        out = torch.empty((n_sel, n_q_heads * head_dim), dtype=q.dtype, device=dev)
    if workspace is None:
        workspace = attn_workspace(n_sel, S, n_q_heads, n_kv_heads, head_dim, dev)
        reuse_plan = False
    with TIMES.span("partial_attn" + timer_tag, dev, 2 if reuse_plan else 3):   # plan, attention, combine
        N.check(N.LIB.cbk_partial_attn(_vp(q), _vp(k_cache), _vp(v_cache), _vp(pos), n_sel, S,
                                       n_q_heads, n_kv_heads, head_dim, float(scale),
                                       dtype_code(q.dtype), _vp(out), _vp(workspace), workspace.numel(),
                                       int(bool(reuse_plan)), _vp(status), _stream(dev)),
                "cbk_partial_attn")
    return out


# ---------------------------------------------------------------------------
# decoder-layer row kernels (RMSNorm with residual add, SiLU * up)
# ---------------------------------------------------------------------------
def add_rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float, delta: torch.Tensor | None = None,
                rows: torch.Tensor | None = None, sum_out: torch.Tensor | None = None,
                out: torch.Tensor | None = None, status=None) -> torch.Tensor:
    """HF RMSNorm of ``s`` = x (rows gathered by ``rows`` when given) plus ``delta``
    (16-bit residual add), in one pass.  ``s`` is written to ``sum_out`` when
    given (it may be ``x`` itself when ``rows`` is None).  x: [..., cols]; the
    result has delta's / the gathered row count and x's last dimension."""
    dev = require_cuda(x, weight, delta, rows, sum_out, out)
    x2 = _rows(x, "x")
    cols = x2.shape[1]
    if weight.dtype != x.dtype or weight.numel() != cols:
        raise ValueError(f"add_rmsnorm: weight must be {x.dtype}[{cols}], got {weight.dtype}{list(weight.shape)}")
    w = weight.contiguous()
    if rows is not None:
        if rows.dtype != torch.int64:
            raise ValueError("add_rmsnorm: rows must be int64")
        rows = rows.contiguous()
        n = rows.numel()
    else:
        n = x2.shape[0]
    d2 = None
    if delta is not None:
        if delta.dtype != x.dtype or delta.shape[-1] != cols or delta.numel() != n * cols:
            raise ValueError(f"add_rmsnorm: delta must be {x.dtype} with {n} rows of {cols}")
        d2 = _rows(delta, "delta")
    lead = (delta.shape[:-1] if delta is not None else
            (x.shape[:-1] if rows is None else (1, n) if x.dim() == 3 else (n,)))
    if out is None:
        out = torch.empty((*lead, cols), dtype=x.dtype, device=dev)
    o2 = out.view(-1, cols)
    s2 = None
    if sum_out is not None:
        if sum_out.dtype != x.dtype or sum_out.numel() != n * cols:
            raise ValueError(f"add_rmsnorm: sum_out must be {x.dtype} with {n} rows of {cols}")
        if rows is not None and sum_out.data_ptr() == x2.data_ptr():
            raise ValueError("add_rmsnorm: sum_out may alias x only without a row gather")
        s2 = sum_out.view(-1, cols)
    with TIMES.span("add_rmsnorm", dev):
        N.check(N.LIB.cbk_add_rmsnorm(_vp(x2), x2.stride(0), x2.shape[0], _vp(rows), _vp(d2),
                                      d2.stride(0) if d2 is not None else 0, _vp(s2),
                                      s2.stride(0) if s2 is not None else 0, _vp(w), float(eps), n, cols,
                                      dtype_code(x.dtype), _vp(o2), o2.stride(0), _vp(status), _stream(dev)),
                "cbk_add_rmsnorm")
    return out


def silu_mul(gate: torch.Tensor, up: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """round16(silu(gate)) * up with the 16-bit roundings of torch's SiLU and mul."""
    dev = require_cuda(gate, up, out)
    if gate.shape != up.shape or gate.dtype != up.dtype:
        raise ValueError(f"silu_mul: gate {gate.dtype}{list(gate.shape)} vs up {up.dtype}{list(up.shape)}")
    g2, u2 = _rows(gate, "gate"), _rows(up, "up")
    if out is None:
        out = torch.empty(gate.shape, dtype=gate.dtype, device=dev)
    o2 = out.view(-1, gate.shape[-1])
    with TIMES.span("silu_mul", dev):
        N.check(N.LIB.cbk_silu_mul(_vp(g2), g2.stride(0), _vp(u2), u2.stride(0), g2.shape[0], g2.shape[1],
                                   dtype_code(gate.dtype), _vp(o2), o2.stride(0), _stream(dev)),
                "cbk_silu_mul")
    return out


def gemv(weight: torch.Tensor, x: torch.Tensor | None = None, gate: torch.Tensor | None = None,
         up: torch.Tensor | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """One-row projection x @ weight.T (a decode step's Linear), fp32 accumulation,
    shape (..., N) for x of shape (..., K) with one row.  With gate and up instead
    of x, the input is round16(round16(silu(gate)) * up) (silu_mul's arithmetic)."""
    src = x if x is not None else gate
    dev = require_cuda(weight, src, up, out)
    if (x is None) == (gate is None) or (gate is None) != (up is None):
        raise ValueError("gemv: pass x, or gate and up")
    k = weight.shape[1]
    if src.shape[-1] != k or src.numel() != k or (up is not None and up.shape != gate.shape):
        raise ValueError(f"gemv: one input row of {k} elements expected, got {list(src.shape)}")
    if weight.stride(1) != 1:
        raise ValueError("gemv: weight rows must be contiguous")
    if out is None:
        out = torch.empty((*src.shape[:-1], weight.shape[0]), dtype=weight.dtype, device=dev)
    xs = [t if t is None or t.is_contiguous() else t.contiguous() for t in (x, gate, up)]
    with TIMES.span("gemv", dev):
        N.check(N.LIB.cbk_gemv(_vp(weight), weight.stride(0), _vp(xs[0]), _vp(xs[1]), _vp(xs[2]), weight.shape[0],
                               k, dtype_code(weight.dtype), _vp(out), _stream(dev)), "cbk_gemv")
    return out


def decode_workspace(cap: int, n_q_heads: int, n_kv_heads: int, head_dim: int, device) -> torch.Tensor:
    """Workspace of decode_attn for a cache of `cap` rows (per-split partial
    results; reusable by calls that do not overlap on the GPU)."""
    n = N.LIB.cbk_decode_attn_workspace_bytes(int(cap), n_q_heads, n_kv_heads, head_dim)
    if n == 0:
        raise ValueError("decode_workspace: bad geometry")
    return torch.zeros((n,), dtype=torch.uint8, device=device)


def decode_attn(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, pos: torch.Tensor,
                n_q_heads: int, n_kv_heads: int, head_dim: int, scale: float, workspace: torch.Tensor,
                out: torch.Tensor | None = None, status=None) -> torch.Tensor:
    """Attention of one query token (q: [n_q_heads * head_dim], rotated) at the
    device position pos (int64, one element) over cache rows 0..pos of
    k_cache / v_cache ([cap][n_kv_heads * head_dim]); returns [1][n_q_heads * head_dim]."""
    dev = require_cuda(q, k_cache, v_cache, pos, workspace)
    if pos.dtype != torch.int64 or pos.numel() != 1:
        raise ValueError("decode_attn: pos must be one int64 on the device")
    if k_cache.shape != v_cache.shape or k_cache.stride() != v_cache.stride() or k_cache.stride(-1) != 1:
        raise ValueError("decode_attn: k_cache and v_cache must have the same row layout")
    qc = q.reshape(-1)
    if not qc.is_contiguous():
        qc = qc.contiguous()
    if out is None:
        out = torch.empty((1, n_q_heads * head_dim), dtype=q.dtype, device=dev)
    with TIMES.span("decode_attn", dev):
        N.check(N.LIB.cbk_decode_attn(_vp(qc), _vp(k_cache), _vp(v_cache), k_cache.stride(0), _vp(pos),
                                      k_cache.shape[0], n_q_heads, n_kv_heads, head_dim, float(scale),
                                      dtype_code(q.dtype), _vp(out), _vp(workspace), workspace.numel(),
                                      _vp(status), _stream(dev)), "cbk_decode_attn")
    return out


def scatter_rows(src: torch.Tensor, idx: torch.Tensor, n_rows: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """Dense [n_rows][...] rows: out[idx[j]] = src[j], zeros elsewhere (idx ascending,
    distinct), every output byte written once."""
    dev = require_cuda(src, idx, out)
    s2 = _rows(src, "src")
    if idx.dtype != torch.int64 or idx.numel() != s2.shape[0]:
        raise ValueError("scatter_rows: idx must be int64 with one entry per source row")
    idx = idx.contiguous()
    if out is None:
        out = torch.empty((n_rows, s2.shape[1]), dtype=src.dtype, device=dev)
    o2 = out.view(-1, s2.shape[1])
    if o2.shape[0] != n_rows:
        raise ValueError(f"scatter_rows: out has {o2.shape[0]} rows, expected {n_rows}")
    row_bytes = s2.shape[1] * s2.element_size()
    with TIMES.span("scatter_rows", dev):
        N.check(N.LIB.cbk_scatter_rows(_vp(s2), s2.stride(0) * s2.element_size(), _vp(idx), idx.numel(), _vp(o2),
                                       o2.stride(0) * o2.element_size(), int(n_rows), row_bytes, _stream(dev)),
                "cbk_scatter_rows")
    return out
