"""KV-head sharding of HKVD on one GPU: each shard's partial deviation comes
from the deviation kernel over its head columns, the partials are combined
with the kernel's pairwise tree (the exchange's combine step), and top-K runs
on the total.  The totals must equal the unsharded kernel's deviations bit for
bit, and the selection the unsharded selection, at 2, 4 and 8 shards.  The
NCCL exchange itself is exercised by the sharded bench workload on 2+ GPUs and
by the gloo tests on CPU."""
import numpy as np
import pytest
import torch

from helpers import to_bits
from oracle import hotpath as hp
from oracle.bf16 import bf16_to_f32

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


@pytest.mark.parametrize("world", [2, 4, 8])
def test_sharded_partials_sum_and_select_like_oracle(world):
    from cacheblend import ops
    from cacheblend.sharding import combine_partials, head_shard
    Hkv, D, lens = 8, 128, [1024, 2048, 1500, 300]
    S = sum(lens)
    g = torch.Generator().manual_seed(world)
    old = (torch.randn((S, Hkv * D), generator=g) * 2).to(torch.bfloat16)
    mask = (torch.rand((S, 1), generator=g) < 0.2).float()
    new = (old.float() + torch.randn((S, Hkv * D), generator=g) * 0.05 * mask).to(torch.bfloat16)
    old_d, new_d = old.to(DEV), new.to(DEV)
    starts = np.cumsum([0] + lens)
    k = hp.topk_count(S, 0.15)
    parts, exp_parts = [], []
    for r in range(world):
        lo, hi = head_shard(Hkv, world, r)
        cols = slice(lo * D, hi * D)
        entries = [{"K": [old_d[a:b, cols].contiguous().unsqueeze(0)],
                    "V": [old_d[a:b, cols].contiguous().unsqueeze(0)]} for a, b in zip(starts, starts[1:])]
        table = ops.ChunkTable(entries, [0], DEV)
        parts.append(ops.kv_deviation_rows(new_d[:, cols].contiguous(), table, 0))
        exp_parts.append(hp.kv_deviation(bf16_to_f32(to_bits(new[:, cols])), bf16_to_f32(to_bits(old[:, cols]))))
    total = combine_partials(parts)
    idx = ops.topk_select(total, k, force_last=True)
    # unsharded: the deviation kernel over all heads, then the same top-K
    entries = [{"K": [old_d[a:b].contiguous().unsqueeze(0)], "V": [old_d[a:b].contiguous().unsqueeze(0)]}
               for a, b in zip(starts, starts[1:])]
    single = ops.kv_deviation_rows(new_d, ops.ChunkTable(entries, [0], DEV), 0)
    idx1 = ops.topk_select(single, k, force_last=True)
    np.testing.assert_array_equal(total.cpu().numpy().view(np.uint32), single.cpu().numpy().view(np.uint32))
    np.testing.assert_array_equal(idx.cpu().numpy(), idx1.cpu().numpy())
    # and both equal the oracle's restatement
    exp_total = hp.tree_sum(np.stack(exp_parts, axis=-1))
    np.testing.assert_array_equal(total.cpu().numpy(), exp_total)
    exp_single = hp.kv_deviation(bf16_to_f32(to_bits(new)), bf16_to_f32(to_bits(old)))
    np.testing.assert_array_equal(exp_total, exp_single)
    np.testing.assert_array_equal(idx.cpu().numpy(), hp.topk_select(exp_single, k, force_last=True))
