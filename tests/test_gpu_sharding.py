"""KV-head sharding of HKVD on one GPU: each shard's partial deviation comes
from the deviation kernel over its head columns, the partials are summed in
rank order (the exchange's combine step), and top-K runs on the total.  The
oracle does the same per-shard fp32 sums: the totals and the selected index
sets must be bit-identical.  The NCCL exchange itself is exercised by the
sharded bench workload on 2+ GPUs and by the gloo tests on CPU."""
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
    exp_total = exp_parts[0].astype(np.float32)
    for p in exp_parts[1:]:
        exp_total = (exp_total + p).astype(np.float32)
    np.testing.assert_array_equal(total.cpu().numpy(), exp_total)
    np.testing.assert_array_equal(idx.cpu().numpy(), hp.topk_select(exp_total, k, force_last=True))
