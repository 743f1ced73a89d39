"""Per-chunk pre-RoPE K / V production (API of cacheblend-hf-v7
``precompute.py``).  A chunk's forward is an ordinary prefill of the HF model;
its outputs are captured with k_proj / v_proj hooks in the layout the blend
kernels read in place: one contiguous (1, Lc, Hkv*D) tensor per layer."""
from __future__ import annotations

import torch

from cacheblend.chunker import Chunk, chunk_offsets, fused_input_ids


def _install_v_proj_hooks(layerwise_model):
    captured: dict[int, torch.Tensor] = {}
    handles = []
    for idx, layer in enumerate(layerwise_model._inner.layers):
        def hook(_m, _inp, out, _idx=idx):
            captured[_idx] = out.detach()
        handles.append(layer.self_attn.v_proj.register_forward_hook(hook))
    return captured, handles


def _forward_capture(layerwise_model, input_ids):
    v_dict, handles = _install_v_proj_hooks(layerwise_model)
    try:
        with torch.inference_mode():
            layerwise_model.forward_layerwise(input_ids=input_ids, use_cache=True)
    finally:
        for h in handles:
            h.remove()
    return v_dict


def precompute_chunk_kv(layerwise_model, chunk: Chunk):
    """Standalone forward of one chunk at positions 0..L-1; returns
    (K_pre_rope per layer, V per layer), each (1, L, Hkv*D)."""
    ids = torch.tensor([chunk.token_ids], dtype=torch.long, device=layerwise_model.device)
    v_dict = _forward_capture(layerwise_model, ids)
    n = layerwise_model.num_layers
    K = [layerwise_model.get_pre_rope_k(i).clone() for i in range(n)]
    V = [v_dict[i].clone() for i in range(n)]
    return K, V


def precompute_chunk_kv_into(layerwise_model, chunk: Chunk, arena):
    """precompute_chunk_kv writing straight into a KVArena slab (one copy of each
    layer's K and V, no intermediate clone); returns the chunk's entry."""
    ids = torch.tensor([chunk.token_ids], dtype=torch.long, device=layerwise_model.device)
    v_dict = _forward_capture(layerwise_model, ids)
    entry = arena.reserve(chunk.chunk_id, len(chunk.token_ids))
    with torch.no_grad():
        for i in range(layerwise_model.num_layers):
            entry["K"][i].copy_(layerwise_model.get_pre_rope_k(i))
            entry["V"][i].copy_(v_dict[i])
    return entry


def precompute_from_cache_prompt(layerwise_model, chunks_in_cache_order, skip_chunk_ids=None):
    """One forward over the whole cache prompt; each chunk's K / V is sliced at
    its position (cross-chunk attention included).  Returns a KVStore."""
    from cacheblend.kv_store import KVStore
    skip = skip_chunk_ids or set()
    ids = fused_input_ids(chunks_in_cache_order, device=layerwise_model.device)
    v_dict = _forward_capture(layerwise_model, ids)
    store = KVStore()
    for chunk, (s, e) in zip(chunks_in_cache_order, chunk_offsets(chunks_in_cache_order)):
        if chunk.chunk_id in skip:
            continue
        K = [layerwise_model.get_pre_rope_k(l)[:, s:e, :].clone() for l in range(layerwise_model.num_layers)]
        V = [v_dict[l][:, s:e, :].clone() for l in range(layerwise_model.num_layers)]
        store.put(chunk.chunk_id, K, V)
    return store
