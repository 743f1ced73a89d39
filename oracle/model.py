"""Oracle restatement of a Mistral/Llama decoder and of the fusion strategies
(numpy fp32, CPU) -- test infrastructure and the timed CPU baseline.

Follows transformers' MistralModel forward (RMSNorm, GQA attention with RoPE,
SiLU-gated MLP) and the reference's fusion functions:
``precompute.py:33-61`` (precompute_chunk_kv), ``fusor.py:25-38``
(fuse_full_recompute) and ``fusor.py:193-497`` (fuse_selective).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from oracle import hotpath as hp


@dataclass
class Config:
    vocab_size: int
    hidden_size: int
    intermediate_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    rope_theta: float
    rms_norm_eps: float

    @classmethod
    def from_hf(cls, c):
        hd = getattr(c, "head_dim", None) or c.hidden_size // c.num_attention_heads
        theta = c.rope_parameters["rope_theta"] if getattr(c, "rope_parameters", None) else c.rope_theta
        return cls(c.vocab_size, c.hidden_size, c.intermediate_size, c.num_hidden_layers,
                   c.num_attention_heads, c.num_key_value_heads, hd, float(theta), c.rms_norm_eps)


class Weights:
    """fp32 numpy copy of an HF causal-LM state dict (Mistral/Llama names)."""

    def __init__(self, sd: dict, cfg: Config, inv_freq=None):
        self.cfg = cfg
        g = lambda n: np.ascontiguousarray(np.asarray(sd[n], np.float32))
        self.embed = g("model.embed_tokens.weight")
        self.lm_head = g("lm_head.weight") if "lm_head.weight" in sd else self.embed
        self.norm = g("model.norm.weight")
        self.layers = []
        for i in range(cfg.num_hidden_layers):
            p = f"model.layers.{i}."
            self.layers.append({k: g(p + n) for k, n in (
                ("q", "self_attn.q_proj.weight"), ("k", "self_attn.k_proj.weight"),
                ("v", "self_attn.v_proj.weight"), ("o", "self_attn.o_proj.weight"),
                ("gate", "mlp.gate_proj.weight"), ("up", "mlp.up_proj.weight"),
                ("down", "mlp.down_proj.weight"), ("ln1", "input_layernorm.weight"),
                ("ln2", "post_attention_layernorm.weight"))})
        self.inv_freq = (np.asarray(inv_freq, np.float32) if inv_freq is not None
                         else hp.inv_freq(cfg.rope_theta, cfg.head_dim))


def rmsnorm(x, w, eps):
    """MistralRMSNorm.forward in fp32: x * rsqrt(mean(x^2) + eps) * w."""
    x = np.asarray(x, np.float32)
    var = np.mean(x * x, axis=-1, keepdims=True, dtype=np.float32)
    return (w * (x / np.sqrt(var + np.float32(eps)))).astype(np.float32)


def mlp(x, L):
    """SiLU-gated MLP; the elementwise SiLU * up runs over row blocks on all
    host cores."""
    from oracle import threads
    g = x @ L["gate"].T
    u = x @ L["up"].T
    a = np.empty_like(g)

    def silu_mul(r0, r1):
        gg = g[r0:r1]
        a[r0:r1] = (gg / (1.0 + np.exp(-gg))).astype(np.float32) * u[r0:r1]

    threads.run([lambda r0=r0, r1=r1: silu_mul(r0, r1) for r0, r1 in threads.row_chunks(g.shape[0])])
    return (a @ L["down"].T).astype(np.float32)


def _heads(x, D):
    return x.reshape(x.shape[0], -1, D)


def rope(x, pos, W: Weights):
    """RoPE in fp32 (the model replay's precision), over row blocks on all host cores."""
    from oracle import threads
    pos = np.asarray(pos)
    parts = threads.run([lambda r0=r0, r1=r1: hp.apply_rope(x[r0:r1], pos[r0:r1], W.inv_freq, W.cfg.head_dim,
                                                            dtype="f32", mode="ref")
                         for r0, r1 in threads.row_chunks(x.shape[0], 256)])
    return np.concatenate(parts, axis=0) if len(parts) > 1 else parts[0]


def attention(q_post, k_post, v, pos_q, W: Weights):
    """GQA causal attention of query rows (positions pos_q, ascending) over all keys."""
    D = W.cfg.head_dim
    o = hp.partial_attention_f32(_heads(q_post, D), _heads(k_post, D), _heads(v, D), pos_q, D ** -0.5)
    return o.astype(np.float32)


def dense_layer(h, L, pos, W: Weights):
    """One full decoder layer; returns (h_out, k_pre, v, k_post)."""
    c = W.cfg
    hn = rmsnorm(h, L["ln1"], c.rms_norm_eps)
    q, k_pre, v = hn @ L["q"].T, hn @ L["k"].T, hn @ L["v"].T
    qp, kp = rope(q, pos, W), rope(k_pre, pos, W)
    a = attention(qp, kp, v, pos, W) @ L["o"].T
    h = (h + a).astype(np.float32)
    h = (h + mlp(rmsnorm(h, L["ln2"], c.rms_norm_eps), L)).astype(np.float32)
    return h, k_pre.astype(np.float32), v.astype(np.float32), kp


def forward_full(ids, W: Weights):
    """Full prefill (fusor.py:25-38 -> model.py forward_layerwise): logits and
    per-layer (pre-RoPE K, V, post-RoPE K)."""
    ids = np.asarray(ids, np.int64)
    pos = np.arange(len(ids))
    h = W.embed[ids]
    kv = []
    for L in W.layers:
        h, kpre, v, kpost = dense_layer(h, L, pos, W)
        kv.append((kpre, v, kpost))
    logits = rmsnorm(h, W.norm, W.cfg.rms_norm_eps) @ W.lm_head.T
    return logits.astype(np.float32), kv


def precompute_chunk_kv(ids, W: Weights):
    """precompute.py:33-61: standalone forward at positions 0..L-1; per-layer
    pre-RoPE K and V of shape (L, Hkv*D)."""
    _, kv = forward_full(ids, W)
    return [k for k, _, _ in kv], [v for _, v, _ in kv]


@dataclass
class SelectiveResult:
    logits: np.ndarray          # (S, vocab), zeros outside the selection (fusor.py:490-491)
    indices: np.ndarray         # (k,) ascending int64
    deviations: np.ndarray      # (S,) check-layer HKVD deviations
    cache_k: list               # per layer (S, Hkv*D) post-RoPE fused K
    cache_v: list               # per layer (S, Hkv*D) fused V


@dataclass
class SelectiveState:
    """Running state of the selective forward after the check layer."""
    S: int
    idx: np.ndarray
    deviations: np.ndarray
    hs: np.ndarray              # (k, hidden) hidden rows of the selected tokens
    K_st: list                  # per layer (S, Hkv*D) concatenated cached pre-RoPE K
    V_st: list
    cache_k: list
    cache_v: list


def selective_begin(chunk_ids, chunk_k, chunk_v, W: Weights, recompute_ratio=0.15, check_layer=1,
                    force_idx=None, n_layers=None) -> SelectiveState:
    """fusor.py:258-406: concat of the cached K/V, the dense layers before the
    check layer, HKVD + force-include, and the check layer itself."""
    prep = selective_prepare(chunk_ids, chunk_k, chunk_v, W, check_layer, n_layers)
    return selective_check(prep, W, recompute_ratio, force_idx)


def selective_prepare(chunk_ids, chunk_k, chunk_v, W: Weights, check_layer=1, n_layers=None) -> dict:
    """First part of selective_begin: the concat of every layer's cached K/V
    (fusor.py:258-272), the embedding and the full layers before the check
    layer (fusor.py:313-323)."""
    ck = check_layer
    nl = W.cfg.num_hidden_layers if n_layers is None else n_layers
    ids = np.concatenate([np.asarray(x, np.int64) for x in chunk_ids])
    S = len(ids)
    pos_full = np.arange(S)
    K_st = [hp.concat_chunks([chunk_k[i][l] for i in range(len(chunk_ids))]) for l in range(nl)]
    V_st = [hp.concat_chunks([chunk_v[i][l] for i in range(len(chunk_ids))]) for l in range(nl)]
    h = W.embed[ids]
    cache_k, cache_v = [], []
    for l in range(ck):
        h, _, v, kpost = dense_layer(h, W.layers[l], pos_full, W)
        cache_k.append(kpost)
        cache_v.append(v)
    return {"S": S, "ck": ck, "h": h, "K_st": K_st, "V_st": V_st, "cache_k": cache_k, "cache_v": cache_v}


def selective_check(prep: dict, W: Weights, recompute_ratio=0.15, force_idx=None) -> SelectiveState:
    """Second part of selective_begin: the check layer (fusor.py:326-406) --
    HKVD on the pre-RoPE K, top-K with force-include, the mixed K/V, the
    selected queries' attention and MLP."""
    c = W.cfg
    S, ck, h, K_st, V_st = prep["S"], prep["ck"], prep["h"], prep["K_st"], prep["V_st"]
    cache_k, cache_v = prep["cache_k"], prep["cache_v"]
    pos_full = np.arange(S)
    L = W.layers[ck]
    hn = rmsnorm(h, L["ln1"], c.rms_norm_eps)
    q, k_pre, v = hn @ L["q"].T, hn @ L["k"].T, hn @ L["v"].T
    dev = hp.kv_deviation(k_pre, K_st[ck])
    if force_idx is None:
        idx = hp.topk_select(dev, hp.topk_count(S, recompute_ratio), force_last=True)
    else:
        idx = np.asarray(force_idx, np.int64)
    k_mixed = hp.scatter_rows(K_st[ck], idx, k_pre[idx])
    v_mixed = hp.scatter_rows(V_st[ck], idx, v[idx])
    qp = rope(q, pos_full, W)
    kp = rope(k_mixed, pos_full, W)
    cache_k.append(kp)
    cache_v.append(v_mixed)
    a = attention(qp[idx], kp, v_mixed, idx, W) @ L["o"].T
    hs = (h[idx] + a).astype(np.float32)
    hs = (hs + mlp(rmsnorm(hs, L["ln2"], c.rms_norm_eps), L)).astype(np.float32)
    return SelectiveState(S, idx, dev, hs, K_st, V_st, cache_k, cache_v)


def selective_layer(st: SelectiveState, l: int, W: Weights, keep_cache: bool = True) -> None:
    """One sparse layer (fusor.py:415-480): selected rows only, attending over
    the full fused cache (RoPE-shifted cached K/V with the fresh rows scattered in)."""
    c = W.cfg
    L = W.layers[l]
    idx = st.idx
    pos_full = np.arange(st.S)
    hn = rmsnorm(st.hs, L["ln1"], c.rms_norm_eps)
    q, k_pre, v = hn @ L["q"].T, hn @ L["k"].T, hn @ L["v"].T
    qp, kp_sparse = rope(q, idx, W), rope(k_pre, idx, W)
    kfull = hp.scatter_rows(rope(st.K_st[l], pos_full, W), idx, kp_sparse)
    vfull = hp.scatter_rows(st.V_st[l], idx, v)
    if keep_cache:
        st.cache_k.append(kfull)
        st.cache_v.append(vfull)
    a = attention(qp, kfull, vfull, idx, W) @ L["o"].T
    hs = (st.hs + a).astype(np.float32)
    st.hs = (hs + mlp(rmsnorm(hs, L["ln2"], c.rms_norm_eps), L)).astype(np.float32)


def selective_end(st: SelectiveState, W: Weights) -> SelectiveResult:
    """fusor.py:483-491: final norm + lm_head on the selected rows, scattered
    into zero logits of the full length."""
    logits_sparse = rmsnorm(st.hs, W.norm, W.cfg.rms_norm_eps) @ W.lm_head.T
    logits = np.zeros((st.S, logits_sparse.shape[1]), np.float32)
    logits[st.idx] = logits_sparse
    return SelectiveResult(logits, st.idx, st.deviations, st.cache_k, st.cache_v)


def fuse_selective(chunk_ids, chunk_k, chunk_v, W: Weights, recompute_ratio=0.15, check_layer=1,
                   force_idx=None, n_layers=None):
    """fusor.py:193-497 for >1 chunk and 0 < ratio < 1 (the selective path).

    chunk_ids: list of per-chunk token id lists; chunk_k / chunk_v: [chunk][layer]
    (Lc, Hkv*D) pre-RoPE K / V.  ``force_idx`` replaces the HKVD selection (to
    compare a device run that selected from its own deviations).  ``n_layers``
    truncates the stack."""
    nl = W.cfg.num_hidden_layers if n_layers is None else n_layers
    st = selective_begin(chunk_ids, chunk_k, chunk_v, W, recompute_ratio, check_layer, force_idx, nl)
    for l in range(check_layer + 1, nl):
        selective_layer(st, l, W)
    return selective_end(st, W)
