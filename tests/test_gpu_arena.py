"""fuse_selective over a KVArena (chunk K/V in one device pool) gives exactly
the plain KVStore's results: same kernels, same bytes; and the arena's
vectorised pointer table equals the per-tensor one."""
import pytest
import torch

from helpers import golden, mock_model

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def test_arena_matches_kvstore_bit_for_bit():
    import cacheblend as cb
    from cacheblend import ops
    model = mock_model(torch.bfloat16, DEV).eval()
    g = golden("mock_fp32.npz")
    ids = [g[f"ids_{i}"].tolist() for i in range(5)]
    lw = cb.LayerwiseModel.from_hf(model)
    chunks = [cb.Chunk(text=f"c{i}", token_ids=t, chunk_id=cb.chunker._stable_id(f"c{i}", t))
              for i, t in enumerate(ids)]
    store = cb.KVStore()
    attn0 = model.model.layers[0].self_attn
    kv_dim = model.config.num_key_value_heads * attn0.head_dim
    arena = cb.KVArena(lw.num_layers, kv_dim, 4096, DEV, dtype=torch.bfloat16)
    for i, c in enumerate(chunks):
        K, V = cb.precompute_chunk_kv(lw, c)
        store.put(c.chunk_id, K, V)
        if i % 2:
            arena.put(c.chunk_id, K, V)                  # copy into the pool
        else:
            cb.precompute_chunk_kv_into(lw, c, arena)      # written in place
    for c in chunks:
        a, b = store.get(c.chunk_id), arena.get(c.chunk_id)
        for l in range(lw.num_layers):
            assert torch.equal(a["K"][l], b["K"][l]) and torch.equal(a["V"][l], b["V"][l])
    # pointer tables: vectorised arena path == per-tensor path
    ents = [arena.get(c.chunk_id) for c in chunks]
    t_fast = ops.ChunkTable(ents, range(1, lw.num_layers), DEV)
    t_slow = ops.ChunkTable([{"K": e["K"], "V": e["V"]} for e in ents], range(1, lw.num_layers), DEV)
    torch.cuda.synchronize()
    assert torch.equal(t_fast.srcs.cpu(), t_slow.srcs.cpu()) and torch.equal(t_fast.starts.cpu(), t_slow.starts.cpu())
    assert t_fast.S == t_slow.S and t_fast.lengths == t_slow.lengths
    # the whole blend
    o1, i1 = cb.fuse_selective(lw, chunks, store, return_layerwise_output=True, return_hkvd_indices=True)
    o2, i2 = cb.fuse_selective(lw, chunks, arena, return_layerwise_output=True, return_hkvd_indices=True)
    torch.cuda.synchronize()
    assert torch.equal(i1, i2)
    assert torch.equal(o1.logits, o2.logits)
    for l in range(lw.num_layers):
        assert torch.equal(o1.past_key_values.layers[l].keys, o2.past_key_values.layers[l].keys)
        assert torch.equal(o1.past_key_values.layers[l].values, o2.past_key_values.layers[l].values)
