"""Multi-GPU partitioning of the blend path.

By request: requests are independent, so each rank (one process per GPU) runs
its own requests end to end with no collective on the data path.

By KV head (long contexts that one GPU cannot hold): rank r of N keeps KV heads
[r*Hkv/N, (r+1)*Hkv/N) and the q heads of their groups.  Concat + RoPE shift,
the fresh-row scatter and partial attention are head-local.  HKVD needs the
per-token deviation summed over all heads: every rank computes its partial
over its own heads, the partials are all-gathered (S fp32 per rank) and
combined on every rank, so every rank selects the identical index set without
a broadcast.

The deviation kernel sums a row as a complete binary tree of pairwise fp32
adds over its 8-element vectors.  A rank's heads are an aligned run of
Hkv*D/(8N) vectors; when that count is a power of two (N a power of two
dividing Hkv, head_dim/8 a power of two) the rank's partial is a node of the
single-GPU tree, and combining the N partials with the same pairwise tree
(``combine_partials``) gives the single-GPU deviations bit for bit: the
selection does not depend on N.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def head_shard(n_kv_heads: int, world: int, rank: int) -> tuple[int, int]:
    """[lo, hi) KV heads of `rank`; heads must divide evenly."""
    if n_kv_heads % world:
        raise ValueError(f"{n_kv_heads} KV heads do not split over {world} ranks")
    per = n_kv_heads // world
    return rank * per, (rank + 1) * per


def combine_partials(parts) -> torch.Tensor:
    """Combine per-rank deviation partials (rank order = head order) with the
    pairwise tree of the deviation kernel: level by level, node = left + right,
    an odd count padded with zeros (adding zero leaves a node unchanged)."""
    level = list(parts)
    if not level:
        raise ValueError("combine_partials: no partials")
    while len(level) > 1:
        nxt = [level[i] + level[i + 1] for i in range(0, len(level) - 1, 2)]
        if len(level) % 2:
            nxt.append(level[-1])
        level = nxt
    return level[0].clone() if level[0] is parts[0] else level[0]


def exchange_deviation(partial: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather per-rank deviation partials (S,) fp32 and combine them with
    the kernel's pairwise tree; every rank returns the same tensor.  Without a process group (one
    GPU) the partial is the total."""
    if not (dist.is_available() and dist.is_initialized()):
        return partial
    world = dist.get_world_size(group)
    if world == 1:
        return partial
    flat = partial.reshape(-1).contiguous()
    gathered = torch.empty((world * flat.numel(),), dtype=flat.dtype, device=flat.device)
    dist.all_gather_into_tensor(gathered, flat, group=group)
    return combine_partials(list(gathered.view(world, -1).unbind(0)))


def sharded_hkvd_select(k_new_shard: torch.Tensor, table_shard, layer: int, k: int, group=None,
                        force_last: bool = True) -> torch.Tensor:
    """HKVD over KV heads spread across ranks: partial deviation of this rank's
    heads (deviation_kernel), exchange, then the same top-K on every rank."""
    from cacheblend import ops
    partial = ops.kv_deviation_rows(k_new_shard, table_shard, layer)
    total = exchange_deviation(partial, group)
    return ops.topk_select(total, k, force_last=force_last)
