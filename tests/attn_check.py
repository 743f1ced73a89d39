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
    ("big_v_f16", 6208, 931, 32, 8, 128, "f16", 4.0, 3e4),
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


def oracle(case, q, k, v, pos, heads=None):
    """(exp, A) of the case from the fp64 oracle."""
    _, S, n_sel, Hq, Hkv, D, dtype, _, _ = case
    return hp.partial_attention(_f32(q, dtype).reshape(n_sel, Hq, D), _f32(k, dtype).reshape(S, Hkv, D),
                                _f32(v, dtype).reshape(S, Hkv, D), pos.numpy(), D ** -0.5,
                                with_abs=True, heads=heads)


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
def plan(pos, n_sel, G, Hkv, sms=148):
    """(C, tile of each selected row, key tiles of each tile) of the partial-
    attention plan: Q tiles of 128/G tokens aligned to the end of the
    selection, paired, and every pair's key range cut into chunks of C
    128-key tiles, C = max(4, ceil(total / SMs))."""
    pos = np.asarray(pos, np.int64)
    tpt = 128 // G
    n_tiles = -(-n_sel // tpt)
    first = n_sel - n_tiles * tpt
    last_tok = np.array([first + (t + 1) * tpt - 1 for t in range(n_tiles)])
    key_tiles = pos[last_tok] // 128 + 1
    n_pairs = (n_tiles + 1) // 2
    later = [2 * p + 1 - (n_tiles & 1) for p in range(n_pairs)]
    total = Hkv * int(key_tiles[later].sum())
    C = max(4, -(-total // sms))
    row_tile = (np.arange(n_sel) - first) // tpt
    return C, row_tile, key_tiles


def planted(case, q, k, v, pos, mistake, heads):
    """The case's attention (fp64) with one planted mistake, for the q heads
    in ``heads``; returns (n, Hq*D) with the other columns zero."""
    _, S, n_sel, Hq, Hkv, D, dtype, _, _ = case
    G = Hq // Hkv
    qf = _f32(q, dtype).reshape(n_sel, Hq, D).astype(np.float64)
    kf = _f32(k, dtype).reshape(S, Hkv, D).astype(np.float64)
    vf = _f32(v, dtype).reshape(S, Hkv, D).astype(np.float64)
    p_ = pos.numpy()
    C, row_tile, key_tiles = plan(p_, n_sel, G, Hkv)
    split_row = key_tiles[row_tile] > C            # the row's tile is split into chunks of C key tiles
    t = np.arange(S)
    out = np.zeros((n_sel, Hq, D))
    for h in heads:
        s = (qf[:, h] @ kf[:, h // G].T) * D ** -0.5
        if mistake == "causal_plus_one":
            vis = t[None, :] <= p_[:, None] + 1
        elif mistake == "causal_minus_one":
            vis = t[None, :] < p_[:, None]
            vis[:, 0] |= p_ == 0
        elif mistake == "drop_split_chunk":
            vis = t[None, :] <= p_[:, None]
            drop = (t[None, :] >= C * 128) & (t[None, :] < 2 * C * 128) & split_row[:, None]
            vis &= ~drop
        elif mistake == "merge_without_max":
            vis = t[None, :] <= p_[:, None]
        else:
            raise ValueError(mistake)
        s = np.where(vis, s, -np.inf)
        if mistake == "merge_without_max":
            # each chunk's O / l from its own max, merged with weights l_c
            # (the 2^(m_c - M) factor left out)
            o = np.zeros((n_sel, D))
            wsum = np.zeros((n_sel, 1))
            for c0 in range(0, S, C * 128):
                sc = s[:, c0:c0 + C * 128]
                m = sc.max(axis=1, keepdims=True)
                ok = np.isfinite(m)
                pc = np.where(ok, np.exp(sc - np.where(ok, m, 0.0)), 0.0)
                l = pc.sum(axis=1, keepdims=True)
                oc = (pc @ vf[c0:c0 + C * 128, h // G]) / np.where(l > 0, l, 1.0)
                o += l * oc
                wsum += l
            exact = np.exp(s - s.max(axis=1, keepdims=True))
            exact = (exact @ vf[:, h // G]) / exact.sum(axis=1, keepdims=True)
            out[:, h] = np.where(split_row[:, None], o / wsum, exact)
        else:
            m = s.max(axis=1, keepdims=True)
            p = np.exp(s - m)
            out[:, h] = (p @ vf[:, h // G]) / p.sum(axis=1, keepdims=True)
    return out.reshape(n_sel, Hq * D)


def round_to(x, dtype):
    """Round fp64/fp32 values to the 16-bit type (what a kernel would store)."""
    return torch.from_numpy(np.asarray(x, np.float32)).to(TDT[dtype]).float().numpy()
