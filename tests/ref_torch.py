"""The reference's selective path (cacheblend-hf-v7 ``fusor.py:258-491``)
restated with stock torch / HF module calls, for the end-to-end tests: run in
bf16 on the GPU it shows what the reference's own 16-bit numerics give on the
same inputs, so our kernels' error against the fp32 oracle can be compared
with the reference's error against it.

Steps as in fusor.py: concat of the stored pre-RoPE K / V (258-272), full
cos/sin (284-286) and an additive causal mask (300-307); full decoder layers
before the check layer (313-323); at the check layer the fresh K / V rows of
the selection scattered into the stored ones (355-361), RoPE of Q and the mixed
K (370-372), the selected query rows against all keys with the mask rows of
the selection and repeat_interleave'd K / V (381-399); after it the selected
rows only, the stored K rotated to the fused positions with the fresh rows
scattered in (415-480); final norm and lm_head on the selected rows (483-484).
The selection is given (the device's own), so both paths attend with the same
rows.
"""
from __future__ import annotations

import sys

import torch
import torch.nn.functional as F


def _heads(x, n, D):
    return x.view(1, x.shape[1], n, D).transpose(1, 2)          # (1, n, T, D)


def selective_logits(model, ids, entries, idx, check_layer):
    """Selected-row logits (k, vocab) of the reference's selective forward."""
    inner = model.model
    cfg = model.config
    L = cfg.num_hidden_layers
    Hq, Hkv = cfg.num_attention_heads, cfg.num_key_value_heads
    D = inner.layers[0].self_attn.head_dim
    G = Hq // Hkv
    rope = sys.modules[type(inner.layers[0].self_attn).__module__].apply_rotary_pos_emb
    dev = inner.embed_tokens.weight.device
    ids = ids.to(dev).view(1, -1)
    S = ids.shape[1]
    idx = idx.to(dev)
    ck = check_layer
    with torch.inference_mode():
        K_st = [torch.cat([e["K"][l] for e in entries], dim=1) for l in range(L)]
        V_st = [torch.cat([e["V"][l] for e in entries], dim=1) for l in range(L)]
        h = inner.embed_tokens(ids)
        cos, sin = inner.rotary_emb(h, torch.arange(S, device=dev).view(1, -1))
        mask = torch.full((S, S), float("-inf"), dtype=h.dtype, device=dev).triu(1).view(1, 1, S, S)

        def attend(layer, q, k, v, m):
            k = k.repeat_interleave(G, dim=1)
            v = v.repeat_interleave(G, dim=1)
            a = F.scaled_dot_product_attention(q, k, v, attn_mask=m, scale=layer.self_attn.scaling)
            return layer.self_attn.o_proj(a.transpose(1, 2).reshape(1, q.shape[2], Hq * D))

        for l in range(ck):
            layer = inner.layers[l]
            hn = layer.input_layernorm(h)
            at = layer.self_attn
            q, k = rope(_heads(at.q_proj(hn), Hq, D), _heads(at.k_proj(hn), Hkv, D), cos, sin)
            h = h + attend(layer, q, k, _heads(at.v_proj(hn), Hkv, D), mask)
            h = h + layer.mlp(layer.post_attention_layernorm(h))
        layer = inner.layers[ck]
        at = layer.self_attn
        hn = layer.input_layernorm(h)
        q, k_pre, v = at.q_proj(hn), at.k_proj(hn), at.v_proj(hn)
        k_mix, v_mix = K_st[ck].clone(), V_st[ck].clone()
        k_mix[:, idx] = k_pre[:, idx]
        v_mix[:, idx] = v[:, idx]
        q, k = rope(_heads(q, Hq, D), _heads(k_mix, Hkv, D), cos, sin)
        msel = mask[:, :, idx, :]
        hs = h[:, idx] + attend(layer, q[:, :, idx], k, _heads(v_mix, Hkv, D), msel)
        hs = hs + layer.mlp(layer.post_attention_layernorm(hs))
        cs, ss = cos[:, idx], sin[:, idx]
        for l in range(ck + 1, L):
            layer = inner.layers[l]
            at = layer.self_attn
            hn = layer.input_layernorm(hs)
            q, k = rope(_heads(at.q_proj(hn), Hq, D), _heads(at.k_proj(hn), Hkv, D), cs, ss)
            _, kf = rope(torch.zeros_like(q[:, :Hkv, :1]).expand(1, Hkv, S, D), _heads(K_st[l], Hkv, D), cos, sin)
            kf = kf.clone()
            kf[:, :, idx] = k
            vf = _heads(V_st[l], Hkv, D).clone()
            vf[:, :, idx] = _heads(at.v_proj(hn), Hkv, D)
            hs = hs + attend(layer, q, kf, vf, msel)
            hs = hs + layer.mlp(layer.post_attention_layernorm(hs))
        return model.lm_head(inner.norm(hs))[0]
