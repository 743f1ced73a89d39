"""Greedy decode over the blended cache (the decode loop of cacheblend-hf-v7's
runners, ``runners.py:106-152``) on the libcbk kernels.

The selective prefill keeps its fused cache with spare rows; each decode step
then runs the decoder for one token at position p: residual add + RMSNorm and
SiLU * up as the fused row kernels, RoPE of the token's Q and K with its K/V
written into cache row p (``rope_scatter`` with one index), and attention of
the one query row over rows [0, p] (``partial_attn``).  Token 1 is the argmax of
the last prefill row, as in the reference; decoding stops after
``max_new_tokens`` tokens or at ``eos_token_id``.
"""
from __future__ import annotations

import torch

from cacheblend import ops
from cacheblend.chunker import Chunk
from cacheblend.fusor import _mlp, _norm, _selective_prefill, fuse_selective
from cacheblend.kv_store import KVStore


def _decode_step(lw, pre, token: torch.Tensor, p: int, status):
    """Logits (vocab,) of one token at position p; its K/V land in cache row p."""
    inner, geo = lw._inner, pre.geo
    device = lw.device
    pos = torch.full((1,), p, dtype=torch.int64, device=device)
    cap = pre.fused_k.shape[1]
    h = inner.embed_tokens(token.view(1, 1))
    m = None
    for li, layer in enumerate(inner.layers):
        attn = layer.self_attn
        hn = _norm(layer.input_layernorm, h, delta=m, sum_out=h if m is not None else None, status=status)
        q, k, v = attn.q_proj(hn), attn.k_proj(hn), attn.v_proj(hn)
        q_rot = ops.rope_scatter(q[0], k[0], v[0], pos, False, cap, geo.n_q, geo.n_kv, geo.head_dim, pre.rope,
                                 pre.fused_k[li], pre.fused_v[li], status=status)
        a = ops.partial_attn(q_rot, pre.fused_k[li, :p + 1], pre.fused_v[li, :p + 1], pos, geo.n_q, geo.n_kv,
                             geo.head_dim, geo.scaling, status=status)
        o = attn.o_proj(a.unsqueeze(0))
        m = _mlp(layer, _norm(layer.post_attention_layernorm, h, delta=o, sum_out=h, status=status))
    return lw.model.lm_head(_norm(inner.norm, h, delta=m, status=status))[0, -1]


def generate_greedy(layerwise_model, chunks: list[Chunk], kv_store: KVStore, max_new_tokens: int,
                    recompute_ratio: float = 0.15, check_layer: int = 1, eos_token_id: int | None = None,
                    rope_mode: str = "ref", status: torch.Tensor | None = None, return_logits: bool = False):
    """CacheBlend selective prefill, then greedy decode over the blended cache.

    Returns the generated token ids (token 1 from the prefill's last row), and
    with ``return_logits`` the logits row that chose each of them.  The
    shortcut cases of fuse_selective (ratio 0, ratio >= 1, one chunk) run the
    reference path: HF prefill and HF decode with ``past_key_values``."""
    if max_new_tokens <= 0:
        return ([], []) if return_logits else []
    lw = layerwise_model
    selective = 0 < recompute_ratio < 1 and len(chunks) > 1
    tokens, rows = [], []
    with torch.inference_mode():
        if not selective:
            out = fuse_selective(lw, chunks, kv_store, recompute_ratio, check_layer, return_layerwise_output=True)
            row = out.logits[0, -1]
            cache = out.past_key_values
            for i in range(max_new_tokens):
                nxt = row.argmax()
                tokens.append(int(nxt.item()))
                rows.append(row)
                if (eos_token_id is not None and tokens[-1] == eos_token_id) or i + 1 == max_new_tokens:
                    break
                step = lw.model(input_ids=nxt.view(1, 1), past_key_values=cache, use_cache=True)
                cache, row = step.past_key_values, step.logits[0, -1]
        else:
            pre = _selective_prefill(lw, chunks, kv_store, recompute_ratio, check_layer, rope_mode, status,
                                     None, extra_tokens=max_new_tokens)
            row = pre.logits[0, -1]
            for i in range(max_new_tokens):
                nxt = row.argmax()
                tokens.append(int(nxt.item()))
                rows.append(row)
                if (eos_token_id is not None and tokens[-1] == eos_token_id) or i + 1 == max_new_tokens:
                    break
                row = _decode_step(lw, pre, nxt, pre.S + i, status)
    return (tokens, rows) if return_logits else tokens
