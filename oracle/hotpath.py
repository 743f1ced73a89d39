"""Oracle restatement of the hot-path functions (numpy, CPU) -- test infrastructure.

Reference files are cited by their path inside cacheblend-hf-v7
(``src/cacheblend/...``); HF transformers functions by module and name.
"""
from __future__ import annotations

import numpy as np

from oracle.bf16 import DECODE, ENCODE, ROUND


# ---------------------------------------------------------------------------
# chunk layout
# ---------------------------------------------------------------------------
def chunk_offsets(lengths):
    """[(start, end)] of each chunk in the fused sequence (chunker.py:68-75)."""
    out, pos = [], 0
    for n in lengths:
        out.append((pos, pos + int(n)))
        pos += int(n)
    return out


def concat_chunks(rows_per_chunk):
    """(a) chunk-KV concat of one layer (fusor.py:258-272): a plain copy into a
    zero-initialised (S, kv_dim) buffer at each chunk's offset.  Works on any
    dtype (uint16 bit patterns for bf16), so it is bit-exact by construction."""
    lens = [r.shape[0] for r in rows_per_chunk]
    offs = chunk_offsets(lens)
    out = np.zeros((offs[-1][1], rows_per_chunk[0].shape[1]), dtype=rows_per_chunk[0].dtype)
    for r, (s, e) in zip(rows_per_chunk, offs):
        out[s:e] = r
    return out


# ---------------------------------------------------------------------------
# RoPE (rope.py:33-64 -> transformers MistralRotaryEmbedding + apply_rotary_pos_emb)
# ---------------------------------------------------------------------------
def inv_freq(theta: float, head_dim: int) -> np.ndarray:
    """MistralRotaryEmbedding.compute_default_rope_parameters:
    1 / theta ** (arange(0, D, 2) / D), evaluated in fp32 like torch does."""
    exps = (np.arange(0, head_dim, 2, dtype=np.int64).astype(np.float32) / np.float32(head_dim))
    return (np.float32(1.0) / np.power(np.float32(theta), exps, dtype=np.float32)).astype(np.float32)


def rope_cos_sin(invf: np.ndarray, positions: np.ndarray, scaling: float = 1.0):
    """cos/sin of angle fp32(inv_freq) * fp32(pos) (MistralRotaryEmbedding.forward:
    the K=1 matmul is one rounded fp32 product).  cos/sin are evaluated in
    float64 and rounded to fp32 (the correctly rounded value; torch/CUDA are
    within an ulp of it).  Returns (len(pos), D/2) fp32 arrays."""
    ang = (invf[None, :].astype(np.float32) * np.asarray(positions).astype(np.float32)[:, None])
    ang = ang.astype(np.float32)
    c = np.cos(ang.astype(np.float64)).astype(np.float32) * np.float32(scaling)
    s = np.sin(ang.astype(np.float64)).astype(np.float32) * np.float32(scaling)
    return c.astype(np.float32), s.astype(np.float32)


def apply_rope(x, positions, invf, head_dim, dtype="bf16", mode="ref", scaling=1.0, cos_sin=None):
    """RoPE of rows ``x`` (n, H*D) at ``positions`` (n,).

    ``x`` holds values of ``dtype`` as float32 (or bit patterns for bf16/f16 if
    given as uint16).  mode="ref" reproduces the 16-bit torch op sequence of
    ``apply_rotary_pos_emb`` (q*cos + rotate_half(q)*sin with cos/sin cast to
    x.dtype, every op rounded); mode="fp32" rotates in fp32 and rounds once.
    ``cos_sin`` (a (n_pos, D/2, 2) fp32 table indexed by position) replaces the
    oracle's own cos/sin, to check rotation arithmetic bit for bit against a
    device table.  Returns float32 values representable in ``dtype``."""
    if x.dtype == np.uint16:
        x = DECODE[dtype](x)
    x = np.asarray(x, np.float32)
    n = x.shape[0]
    H = x.shape[1] // head_dim
    half = head_dim // 2
    xh = x.reshape(n, H, head_dim)
    lo, hi = xh[..., :half], xh[..., half:]
    if cos_sin is None:
        c, s = rope_cos_sin(invf, positions, scaling)
    else:
        tab = np.asarray(cos_sin, np.float32)[np.asarray(positions, np.int64)]
        c, s = tab[..., 0], tab[..., 1]
    c, s = c[:, None, :], s[:, None, :]
    rnd = ROUND[dtype]
    if mode == "ref":
        c, s = rnd(c), rnd(s)
        out_lo = rnd(rnd(lo * c) - rnd(hi * s))
        out_hi = rnd(rnd(hi * c) + rnd(lo * s))
    else:
        out_lo = rnd((lo * c).astype(np.float32) - (hi * s).astype(np.float32))
        out_hi = rnd((hi * c).astype(np.float32) + (lo * s).astype(np.float32))
    return np.concatenate([out_lo, out_hi], axis=-1).reshape(n, H * head_dim).astype(np.float32)


def apply_rope_f64(x, positions, invf, head_dim):
    """Exact-math RoPE (float64) -- the yardstick for the fp32 mode."""
    x = np.asarray(x, np.float64)
    n = x.shape[0]
    H = x.shape[1] // head_dim
    half = head_dim // 2
    xh = x.reshape(n, H, head_dim)
    ang = (invf[None, :].astype(np.float32) * np.asarray(positions).astype(np.float32)[:, None])
    c = np.cos(ang.astype(np.float64))[:, None, :]
    s = np.sin(ang.astype(np.float64))[:, None, :]
    lo, hi = xh[..., :half], xh[..., half:]
    return np.concatenate([lo * c - hi * s, hi * c + lo * s], axis=-1).reshape(n, H * head_dim)


# ---------------------------------------------------------------------------
# HKVD (hkvd.py:23-77) and the force-include rule (fusor.py:344-353)
# ---------------------------------------------------------------------------
def kv_deviation(k_new, k_old, order="kernel"):
    """dev[t] = sum_f (K_new - K_old)^2 in fp32 (hkvd.py:42-51).

    order="kernel": the fixed order of the CUDA kernel, reproduced exactly:
      each 8-element vector's squares are summed in element order
      (s = d0*d0, then s = s + de*de, separately rounded fp32 ops); the row
      total is the complete binary tree of pairwise adds over the vector
      sums, zero-padded to a power of two.  An aligned power-of-two slice of
      the features (a shard's KV heads) is a subtree of it.
    order="f64": float64 sum rounded to fp32 (an order-free yardstick)."""
    a = np.asarray(k_new, np.float32)
    b = np.asarray(k_old, np.float32)
    if a.shape != b.shape:
        raise ValueError(f"shape mismatch: K_new={a.shape}, K_old={b.shape}")
    if a.ndim == 3:
        if a.shape[0] != 1:
            raise NotImplementedError("kv_deviation: batch>1 not supported")
        a, b = a[0], b[0]
    elif a.ndim != 2:
        raise ValueError(f"unsupported ndim: {a.ndim}")
    d = (a - b).astype(np.float32)
    if order == "f64":
        return np.sum(d.astype(np.float64) ** 2, axis=1).astype(np.float32)
    S, F = d.shape
    assert F % 8 == 0
    sq = (d * d).astype(np.float32).reshape(S, F // 8, 8)
    vec = sq[:, :, 0].copy()
    for e in range(1, 8):
        vec = (vec + sq[:, :, e]).astype(np.float32)
    return tree_sum(vec)


def tree_sum(x):
    """Complete binary tree of pairwise fp32 adds along the last axis (zero-padded
    to a power of two; adjacent nodes paired level by level)."""
    x = np.asarray(x, np.float32)
    n = x.shape[-1]
    p = 1
    while p < n:
        p *= 2
    if p != n:
        x = np.concatenate([x, np.zeros(x.shape[:-1] + (p - n,), np.float32)], axis=-1)
    while x.shape[-1] > 1:
        x = (x[..., 0::2] + x[..., 1::2]).astype(np.float32)
    return x[..., 0].copy()


def topk_count(S: int, ratio: float) -> int:
    """hkvd.py:70-73: k = max(1, min(S, int(S * ratio)))."""
    return max(1, min(S, int(S * ratio)))


def _order_keys(dev):
    u = np.asarray(dev, np.float32).view(np.uint32)
    return np.where(u & np.uint32(0x80000000), ~u, u | np.uint32(0x80000000)).astype(np.uint32)


def topk_select(dev, k, force_last=False):
    """select_top_k (hkvd.py:58-77) with k given, then optionally the
    force-include rule (fusor.py:344-353).  Ties at the k-th value are broken
    lowest index first (torch.topk leaves this unspecified).  NaN ranks highest
    (torch.topk semantics)."""
    dev = np.asarray(dev, np.float32)
    S = dev.shape[0]
    keys = _order_keys(dev)
    order = np.lexsort((np.arange(S), -keys.astype(np.int64)))   # key desc, index asc
    idx = np.sort(order[:k])
    if force_last and (S - 1) not in set(idx.tolist()):
        # drop the selected element of minimal deviation (first occurrence, as argmin does)
        sel_keys = keys[idx]
        drop = idx[int(np.argmin(sel_keys))]
        idx = np.sort(np.concatenate([idx[idx != drop], [S - 1]]))
    return idx.astype(np.int64)


def select_top_k(dev, ratio):
    return topk_select(dev, topk_count(len(dev), ratio), force_last=False)


def force_include_last(idx, dev):
    """fusor.py:344-353 on an existing selection."""
    S = len(dev)
    idx = np.asarray(idx, np.int64)
    if (S - 1) in set(idx.tolist()):
        return idx
    sel = np.asarray(dev, np.float32)[idx]
    drop = idx[int(np.argmin(sel))]
    return np.sort(np.concatenate([idx[idx != drop], [S - 1]])).astype(np.int64)


# ---------------------------------------------------------------------------
# scatter (fusor.py:355-361, 449-458) and partial attention (381-399, 462-474)
# ---------------------------------------------------------------------------
def scatter_rows(cache, idx, fresh):
    """fused[idx] = fresh, cached rows elsewhere (bit-exact copy)."""
    out = np.array(cache, copy=True)
    out[np.asarray(idx, np.int64)] = fresh
    return out


def partial_attention(q, k, v, pos, scale, dtype=np.float64, with_abs=False, heads=None):
    """softmax(scale * Q_sel K^T + causal(pos)) V with GQA (n_rep = Hq / Hkv).

    q: (n, Hq, D); k, v: (S, Hkv, D); pos: (n,) ascending.  Returns (n, Hq*D).
    Keys t > pos[j] are excluded, like the -inf rows of the reference mask
    (fusor.py:301-307, 385).

    with_abs=True also returns the same softmax weights applied to |V|
    (sum_t p_t |v_t| / sum_t p_t), the scale that 16-bit rounding of P and of
    the output acts on: an error bound for a 16-bit kernel is a fraction of
    it.  ``heads`` restricts the computation to those q heads (the other
    columns are left zero)."""
    q = np.asarray(q, dtype)
    k = np.asarray(k, dtype)
    v = np.asarray(v, dtype)
    n, Hq, D = q.shape
    S, Hkv, _ = k.shape
    G = Hq // Hkv
    out = np.zeros((n, Hq, D), dtype)
    absm = np.zeros((n, Hq, D), dtype) if with_abs else None
    pos = np.asarray(pos, np.int64)
    t = np.arange(S)
    for h in (range(Hq) if heads is None else heads):
        kh, vh = k[:, h // G, :], v[:, h // G, :]
        s = (q[:, h, :] @ kh.T) * scale                       # (n, S)
        s = np.where(t[None, :] <= pos[:, None], s, -np.inf)
        m = s.max(axis=1, keepdims=True)
        p = np.exp(s - m)
        l = p.sum(axis=1, keepdims=True)
        out[:, h, :] = (p @ vh) / l
        if with_abs:
            absm[:, h, :] = (p @ np.abs(vh)) / l
    if with_abs:
        return out.reshape(n, Hq * D), absm.reshape(n, Hq * D)
    return out.reshape(n, Hq * D)


def partial_attention_f32(q, k, v, pos, scale):
    """fp32 partial_attention for the model replay: the same softmax attention,
    computed per (q head, block of query rows) on all host cores; a block's
    keys stop at its largest position (keys past it are masked for every row
    of the block).  q: (n, Hq, D); k, v: (S, Hkv, D); pos ascending.  Returns
    (n, Hq*D) fp32."""
    from oracle import threads
    q = np.asarray(q, np.float32)
    k = np.asarray(k, np.float32)
    v = np.asarray(v, np.float32)
    n, Hq, D = q.shape
    Hkv = k.shape[1]
    G = Hq // Hkv
    pos = np.asarray(pos, np.int64)
    out = np.empty((n, Hq, D), np.float32)
    kh = [np.ascontiguousarray(k[:, g, :]) for g in range(Hkv)]
    vh = [np.ascontiguousarray(v[:, g, :]) for g in range(Hkv)]
    rb = 256

    def block(h, r0, r1):
        pm = int(pos[r0:r1].max()) + 1
        s = (q[r0:r1, h, :] @ kh[h // G][:pm].T) * np.float32(scale)
        s[np.arange(pm)[None, :] > pos[r0:r1, None]] = -np.inf
        s -= s.max(axis=1, keepdims=True)
        np.exp(s, out=s)
        out[r0:r1, h, :] = (s @ vh[h // G][:pm]) / s.sum(axis=1, keepdims=True)

    threads.run([lambda h=h, r0=r0: block(h, r0, min(n, r0 + rb)) for h in range(Hq) for r0 in range(0, n, rb)])
    return out.reshape(n, Hq * D)


def encode(x, dtype):
    return ENCODE[dtype](x)


def decode(x, dtype):
    return DECODE[dtype](x)
