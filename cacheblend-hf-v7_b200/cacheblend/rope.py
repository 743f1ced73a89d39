"""RoPE shift of pre-RoPE K (API of cacheblend-hf-v7 ``rope.py``) on the
sm_100a row kernel: one pass over the rows, rotation in fp32 registers."""
from __future__ import annotations

import torch

from cacheblend import ops


def rope_table_for(layerwise_model, n_pos: int, device: torch.device) -> torch.Tensor:
    """Cached cos/sin table of the model for positions [0, n_pos); grown on demand."""
    cache = getattr(layerwise_model, "_cbk_rope_tables", None)
    if cache is None:
        cache = {}
        try:
            layerwise_model._cbk_rope_tables = cache
        except AttributeError:
            pass
    rot = layerwise_model._inner.rotary_emb
    key = (str(device), float(getattr(rot, "attention_scaling", 1.0)))
    tab = cache.get(key)
    if tab is None or tab.shape[0] < n_pos:
        n = max(int(n_pos), 1)
        n = 1 << (n - 1).bit_length() if n > 1024 else 1024      # grow geometrically
        tab = ops.rope_table(rot.inv_freq.to(device), n, float(getattr(rot, "attention_scaling", 1.0)))
        cache[key] = tab
    return tab


def apply_rope_shift(K_pre_rope: torch.Tensor, target_positions: torch.Tensor,
                     layerwise_model, status: torch.Tensor | None = None) -> torch.Tensor:
    """RoPE of pre-RoPE K (B, S, Hkv*D) at absolute ``target_positions`` (B, S);
    same shape and dtype out -- reference rope.py:33-64 (HF apply_rotary_pos_emb
    numerics, reproduced by CBK_ROPE_REF).

    Positions on the host are checked on the host (ValueError when negative)
    and size the cos/sin table.  Positions on the device are never read back:
    the table covers the model's ``max_position_embeddings`` (or more, if a
    larger one is cached), and a position outside it -- or negative -- sets
    CBK_STATUS_BAD_INDEX in ``status`` (int32 CUDA tensor, optional) and leaves
    that row of the result unwritten."""
    attn0 = layerwise_model._inner.layers[0].self_attn
    head_dim = attn0.head_dim
    B, S, F = K_pre_rope.shape
    ops.require_cuda(K_pre_rope)
    if target_positions.numel() != B * S:
        raise ValueError(f"target_positions {tuple(target_positions.shape)} must be (B, S) = ({B}, {S})")
    if target_positions.device.type == "cpu":
        host = target_positions.reshape(-1).to(torch.int64)
        if host.numel() and int(host.min()) < 0:
            raise ValueError("negative target position")
        n_pos = int(host.max()) + 1 if host.numel() else 1
        pos = host.to(K_pre_rope.device, non_blocking=True)
    else:
        pos = target_positions.to(device=K_pre_rope.device, dtype=torch.int64).reshape(-1)
        cfg = getattr(getattr(layerwise_model, "model", None), "config", None)
        n_pos = int(getattr(cfg, "max_position_embeddings", 0) or 0) or 32768
    table = rope_table_for(layerwise_model, n_pos, K_pre_rope.device)
    out = ops.rope_rows(K_pre_rope, pos, table, head_dim, mode="ref", status=status)
    return out.view(B, S, F)
