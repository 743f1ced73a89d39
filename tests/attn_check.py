"""Partial-attention parity: the inputs of the GPU cases, the error bound they
are held to, and planted mistakes that the bound must catch.

Bound, element by element:

    |got - exp| <= tol * (|exp| + A),   A = sum_t p_t |v_t| / sum_t p_t

``exp`` is the exact (fp64) softmax attention of the same 16-bit inputs and
``A`` the same softmax weights applied to |V| (both from the oracle).  The
kernel rounds P to the 16-bit type before P V (relative error 2^-9 in bf16 on
each p: at most 2^-9 A on the output, and 2^-9 |exp| through the fp32 row
sum), stores split partials O/l in the 16-bit type (2^-9 A) and rounds the
output once (2^-9 |exp|): 2^-8 (|exp| + A) in all, so tol = 2^-7 (bf16)
leaves a factor of two; fp16 has 2^-11 steps and tol = 2^-9.  The bound
scales with the output itself, so it is as tight on a flat softmax over
thousands of keys (outputs ~0.02) as on a peaked one (outputs ~1).

``planted`` computes the attention with one mistake a kernel could make (a
causal bound one key too far, a split chunk of keys left out, split partials
merged without their max correction); ``tests/test_attn_bound.py`` shows that
each one violates the bound on the peaked cases, on the CPU.
"""
from __future__ import annotations

import math

import numpy as np
import torch

from oracle import hotpath as hp
from oracle.bf16 import bf16_to_f32, f16_to_f32

TOL = {"bf16": 2.0 ** -7, "f16": 2.0 ** -9}
DEC = {"bf16": bf16_to_f32, "f16": f16_to_f32}
TDT = {"bf16": torch.bfloat16, "f16": torch.float16}

# name, S, n_sel, Hq, Hkv, D, dtype, q scale, v scale
CASES = [
    ("mistral7k", 6208, 931, 32, 8, 128, "bf16", 1.0, 1.0),
    ("mistral7k_peaked", 6208, 931, 32, 8, 128, "bf16", 8.0, 1.0),
    ("mock", 544, 81, 4, 2, 64, "bf16", 1.0, 1.0),
    ("dense_causal", 300, 300, 8, 2, 128, "bf16", 1.0, 1.0),
    ("dense_4k_peaked", 4096, 4096, 32, 8, 128, "bf16", 4.0, 1.0),
    ("g1", 1000, 150, 8, 8, 128, "bf16", 1.0, 1.0),
    ("g8", 2048, 200, 64, 8, 128, "bf16", 1.0, 1.0),
    ("g8_peaked", 2048, 200, 64, 8, 128, "bf16", 6.0, 1.0),
    ("g16", 700, 33, 16, 1, 64, "f16", 1.0, 1.0),
    ("short", 100, 15, 4, 1, 128, "bf16", 1.0, 1.0),
    ("one_row", 2000, 1, 8, 2, 128, "bf16", 1.0, 1.0),
    ("f16_128", 1500, 225, 32, 8, 128, "f16", 1.0, 1.0),
    ("long_split", 20000, 2000, 32, 8, 128, "bf16", 1.0, 1.0),
    ("long_split_peaked", 20000, 2000, 32, 8, 128, "bf16", 4.0, 1.0),
    ("big_v_split", 20000, 2000, 32, 8, 128, "bf16", 1.0, 1e5),
    ("big_v_f16", 6208, 931, 32, 8, 128, "f16", 4.0, 1e4),   # |V| up to ~5.5e4 (fp16 max 65504)
]
CASE = {c[0]: c for c in CASES}


def make_inputs(case):
    """Seeded 16-bit q [n][Hq*D], k, v [S][Hkv*D] (CPU tensors) and ascending
    positions (the last one S - 1, like a blended prefill's selection)."""
    name, S, n_sel, Hq, Hkv, D, dtype, qs, vs = case
    g = torch.Generator().manual_seed(S + n_sel + int(qs * 10) + (7 if vs != 1.0 else 0))
    if n_sel == S:
        pos = torch.arange(S)
    else:
        pos = torch.sort(torch.randperm(S - 1, generator=g)[: n_sel - 1]).values
        pos = torch.cat([pos, torch.tensor([S - 1])])
    q = (torch.randn((n_sel, Hq * D), generator=g) * qs).to(TDT[dtype])
    k = torch.randn((S, Hkv * D), generator=g).to(TDT[dtype])
    v = (torch.randn((S, Hkv * D), generator=g) * vs).to(TDT[dtype])
    return q, k, v, pos


def _f32(t, dtype):
    return DEC[dtype](t.contiguous().view(torch.int16).numpy().view(np.uint16))


def oracle(case, q, k, v, pos, heads=None, rows=None):
    """(exp, A) of the case from the fp64 oracle (of the selected rows ``rows``
    only when given: query rows are independent)."""
    _, S, n_sel, Hq, Hkv, D, dtype, _, _ = case
    rows = np.arange(n_sel) if rows is None else np.asarray(rows)
    qf = _f32(q, dtype).reshape(n_sel, Hq, D)[rows]
    return hp.partial_attention(qf, _f32(k, dtype).reshape(S, Hkv, D), _f32(v, dtype).reshape(S, Hkv, D),
                                pos.numpy()[rows], D ** -0.5, with_abs=True, heads=heads)


def violations(got, exp, absm, dtype, cols=None):
    """(count of elements outside the bound, worst |err| / (|exp| + A)) of got vs exp."""
    got = np.asarray(got, np.float64)
    if cols is not None:
        got, exp, absm = got[:, cols], exp[:, cols], absm[:, cols]
    if not np.isfinite(got).all():
        return got.size, math.inf
    ratio = np.abs(got - exp) / (np.abs(exp) + absm + 1e-300)
    return int((ratio > TOL[dtype]).sum()), float(ratio.max())


def check(got, exp, absm, dtype):
    """Assert the bound (and the scale-relative summary figures)."""
    got = np.asarray(got, np.float64)
    assert np.isfinite(got).all(), "non-finite attention output"
    n_bad, worst = violations(got, exp, absm, dtype)
    err = np.abs(got - exp)
    scale = float(np.abs(exp).max())
    detail = (f"{n_bad} elements outside tol*(|exp|+A) (tol {TOL[dtype]:.2e}, worst ratio {worst:.3e}); "
              f"max|err| {err.max():.3e}, max|exp| {scale:.3e}")
    assert n_bad == 0, detail
    assert err.max() <= 2e-2 * max(scale, 1e-30), detail
    return worst


# ---------------------------------------------------------------------------
# the kernel's split plan (attn_plan_kernel restated) and planted mistakes
# ---------------------------------------------------------------------------
PLAN_ITEM_COST = 2      # the kernel's CBK_ATTN_ITEM_COST
PLAN_DYN_PCT = 0        # the kernel's CBK_ATTN_DYN_PCT


def plan(pos, n_sel, G, Hkv, sms=148, c0=PLAN_ITEM_COST, dyn=PLAN_DYN_PCT):
    """The partial-attention work plan (attn_plan_kernel restated): Q tiles of
    128/G tokens aligned to the end of the selection, paired; a pair's steps
    are its later tile's 128-key tiles, and every item costs c0 steps more.
    Small units (longest + c0 at most half an SM's share) are whole items;
    otherwise the shortest pairs' units (about ``dyn`` % of the cost) are
    whole items of a dynamic tail, and the other units, each c0 of cost then
    its steps, are laid end to end and cut into ``sms`` equal ranges of cost;
    a unit whose steps cross a cut is split there.  Returns (tile of each selected row, pair of each
    tile, cuts) with cuts[(h, pair)] the key-tile indices where that unit is
    split (empty when it is not)."""
    pos = np.asarray(pos, np.int64)
    tpt = 128 // G
    n_tiles = -(-n_sel // tpt)
    first = n_sel - n_tiles * tpt
    key_tiles = np.array([pos[first + (t + 1) * tpt - 1] // 128 + 1 for t in range(n_tiles)])
    n_pairs = (n_tiles + 1) // 2
    odd = n_tiles & 1
    later = [2 * p + 1 - odd for p in range(n_pairs)]
    L = key_tiles[later]
    Wh = int(L.sum())
    W = Hkv * Wh
    n_units = Hkv * n_pairs
    Wc = W + c0 * n_units
    B = min(W, sms)
    off = np.concatenate([[0], np.cumsum(L)])
    cuts = {(h, p): [] for h in range(Hkv) for p in range(n_pairs)}
    if (int(L.max()) + c0) * 2 * B > Wc:
        budget = dyn * Wc // 100
        p_cut = max([0] + [p for p in range(1, n_pairs) if Hkv * (int(off[p]) + c0 * p) <= budget])
        n_ps = n_pairs - p_cut
        Wh_s = Wh - int(off[p_cut])
        Wc_s = Hkv * Wh_s + c0 * Hkv * n_ps
        B_s = min(Hkv * Wh_s, sms)
        starts = [w * Wc_s // B_s for w in range(B_s + 1)]
        for h in range(Hkv):
            for p in range(p_cut, n_pairs):
                Q = (h * n_ps + (p - p_cut) + 1) * c0 + h * Wh_s + int(off[p]) - int(off[p_cut])
                cuts[(h, p)] = [s_ - Q for s_ in starts if Q < s_ < Q + int(L[p])]
    row_tile = (np.arange(n_sel) - first) // tpt
    tile_pair = (np.arange(n_tiles) + odd) // 2
    return row_tile, tile_pair, cuts


def planted(case, q, k, v, pos, mistake, heads, rows=None):
    """The case's attention (fp64) with one planted mistake, for the q heads
    in ``heads`` (and the selected rows ``rows`` when given); returns
    (rows, Hq*D) with the other columns zero.  The split
    mistakes act on the kernel's own pieces (``plan``): "drop_split_chunk"
    leaves out a split row's second piece of keys, "merge_without_max" merges
    the pieces' O / l with weights l_c, without the 2^(m_c - M) correction."""
    _, S, n_sel, Hq, Hkv, D, dtype, _, _ = case
    G = Hq // Hkv
    qf = _f32(q, dtype).reshape(n_sel, Hq, D).astype(np.float64)
    kf = _f32(k, dtype).reshape(S, Hkv, D).astype(np.float64)
    vf = _f32(v, dtype).reshape(S, Hkv, D).astype(np.float64)
    row_tile, tile_pair, cuts = plan(pos.numpy(), n_sel, G, Hkv)
    rows = np.arange(n_sel) if rows is None else np.asarray(rows)
    p_ = pos.numpy()[rows]
    qf = qf[rows]
    n_r = len(rows)
    t = np.arange(S)
    out = np.zeros((n_r, Hq, D))
    for h in heads:
        kvh = h // G
        # key bounds of each row's pieces: [0, c1, c2, ..., end) in keys
        bounds = [[0] + [c * 128 for c in cuts[(kvh, tile_pair[row_tile[j]])]] + [S] for j in rows]
        s = (qf[:, h] @ kf[:, kvh].T) * D ** -0.5
        if mistake == "causal_plus_one":
            vis = t[None, :] <= p_[:, None] + 1
        elif mistake == "causal_minus_one":
            vis = t[None, :] < p_[:, None]
            vis[:, 0] |= p_ == 0
        elif mistake in ("drop_split_chunk", "merge_without_max"):
            vis = t[None, :] <= p_[:, None]
            if mistake == "drop_split_chunk":
                for j, b in enumerate(bounds):
                    if len(b) > 2:
                        vis[j, b[1]:b[2]] = False
        else:
            raise ValueError(mistake)
        s = np.where(vis, s, -np.inf)
        m = s.max(axis=1, keepdims=True)
        p = np.exp(s - m)
        exact = (p @ vf[:, kvh]) / p.sum(axis=1, keepdims=True)
        if mistake == "merge_without_max":
            for j, b in enumerate(bounds):
                if len(b) <= 2:
                    continue
                o, wsum = np.zeros(D), 0.0
                for a, e in zip(b[:-1], b[1:]):
                    sc = s[j, a:e]
                    if not np.isfinite(sc).any():
                        continue
                    pc = np.exp(sc - sc.max())
                    l = pc.sum()
                    o += l * ((pc @ vf[a:e, kvh]) / l)
                    wsum += l
                exact[j] = o / wsum
        out[:, h] = exact
    return out.reshape(n_r, Hq * D)


def in_place_masked(case, q, k, v, pos, heads, rows=None):
    """The case's attention (fp64) as the kernel forms it on diagonal key tiles:
    the scores of keys past a row's position are set to -inf and the tile runs the
    full-tile code, whose polynomial exponentials clamp the argument at -126, so a
    masked key in a polynomial slot weighs 2^-126 (ex2.approx gives 0).  Here every
    masked key of the key tiles the row's Q tile visits gets 2^-126 (an upper bound
    on the kernel's residual).  Split rows are formed per piece of the kernel's plan
    and merged as attn_combine_kernel does (w = l 2^(m - M)); a piece in which the
    row sees no key has m = -inf and weight 0."""
    _, S, n_sel, Hq, Hkv, D, dtype, _, _ = case
    G = Hq // Hkv
    qf = _f32(q, dtype).reshape(n_sel, Hq, D).astype(np.float64)
    kf = _f32(k, dtype).reshape(S, Hkv, D).astype(np.float64)
    vf = _f32(v, dtype).reshape(S, Hkv, D).astype(np.float64)
    row_tile, tile_pair, cuts = plan(pos.numpy(), n_sel, G, Hkv)
    tpt = 128 // G
    n_tiles = -(-n_sel // tpt)
    first = n_sel - n_tiles * tpt
    pos_np = pos.numpy()
    rows = np.arange(n_sel) if rows is None else np.asarray(rows)
    out = np.zeros((len(rows), Hq, D))
    lg2 = math.log2(math.e)
    for h in heads:
        kvh = h // G
        for r, j in enumerate(rows):
            t = row_tile[j]
            end = (pos_np[min(first + (t + 1) * tpt, n_sel) - 1] // 128 + 1) * 128   # keys the tile visits
            end = min(end, S)
            x = (kf[:end, kvh] @ qf[j, h]) * D ** -0.5 * lg2                    # log2 units
            vis = np.arange(end) <= pos_np[j]
            # the pair's cuts are in its later tile's key tiles: pieces past this tile's
            # last key tile hold none of its keys
            bounds = [0] + [min(c * 128, end) for c in cuts[(kvh, tile_pair[t])]] + [end]
            ms, ls, os_ = [], [], []
            for a, e in zip(bounds[:-1], bounds[1:]):
                if a >= e:
                    continue
                xv, sv = x[a:e], vis[a:e]
                m = xv[sv].max() if sv.any() else -np.inf
                p = np.where(sv, np.exp2(xv - (m if np.isfinite(m) else 0.0)), 2.0 ** -126)
                l = p.sum()
                ms.append(m)
                ls.append(l)
                os_.append((p @ vf[a:e, kvh]) / l)
            M = max(ms)
            w = np.array([l * 2.0 ** (m - M) if np.isfinite(m) else 0.0 for m, l in zip(ms, ls)])
            out[r, h] = (w[:, None] * np.array(os_)).sum(axis=0) / w.sum()
    return out.reshape(len(rows), Hq * D)


def round_to(x, dtype):
    """Round fp64/fp32 values to the 16-bit type (what a kernel would store)."""
    return torch.from_numpy(np.asarray(x, np.float32)).to(TDT[dtype]).float().numpy()
