"""CUDA graphs of the selective path.

BlendGraph (fuse_selective captured as one CUDA graph) gives the eager path's
logits and selection bit for bit, also for other chunks of the same lengths
after the chunk table and ids are refreshed, and after a chunk is stored
again under the same id (new tensors: the table follows their addresses, not
object identities).  fuse_selective replays a cached graph by default: its
results equal the eager path's (cuda_graph=False), each call returns new
tensors, and logits_rows="last" returns the dense path's last row bit for bit."""
import pytest
import torch

from test_gpu_fusor import _setup

pytestmark = pytest.mark.gpu

CFG_D128 = dict(vocab_size=2000, hidden_size=1024, intermediate_size=2048, num_hidden_layers=4,
                num_attention_heads=8, num_key_value_heads=2, head_dim=128, rope_theta=1e6, rms_norm_eps=1e-5,
                max_position_embeddings=8192, sliding_window=None)


def _other_chunks(cb, lw, chunks, store, seed):
    g = torch.Generator().manual_seed(seed)
    vocab = lw.model.config.vocab_size
    new = []
    for i, c in enumerate(chunks):
        t = torch.randint(0, vocab, (c.length,), generator=g).tolist()
        nc = cb.Chunk(text=f"o{seed}_{i}", token_ids=t, chunk_id=cb.chunker._stable_id(f"o{seed}_{i}", t))
        K, V = cb.precompute_chunk_kv(lw, nc)
        store.put(nc.chunk_id, K, V)
        new.append(nc)
    return new


def _eager(cb, lw, chunks, store, **kw):
    return cb.fuse_selective(lw, chunks, store, recompute_ratio=0.15, check_layer=1, return_hkvd_indices=True,
                             cuda_graph=False, **kw)


@pytest.mark.parametrize("cfg", [None, CFG_D128])
def test_blend_graph_matches_eager(cfg):
    if cfg is None:
        cb, lw, model, chunks, store = _setup()
    else:
        cb, lw, model, chunks, store = _setup(cfg, n_chunks=6, chunk_len=300, q_len=40, seed=3)
    bg = cb.BlendGraph(lw, chunks, store, recompute_ratio=0.15, check_layer=1)
    for reqs in (chunks, _other_chunks(cb, lw, chunks, store, 11), chunks):
        ref, ref_idx = _eager(cb, lw, reqs, store)
        got = bg(reqs, store)
        torch.cuda.synchronize()
        assert torch.equal(bg.idx, ref_idx)
        assert torch.equal(got, ref)
    with pytest.raises(ValueError):
        bg(chunks[:-1], store)


def test_graph_sees_a_restored_chunk():
    """A chunk evicted and stored again under the same id (new K/V values) is
    read from its new tensors by the next replay."""
    cb, lw, model, chunks, store = _setup(CFG_D128, n_chunks=6, chunk_len=300, q_len=40, seed=3)
    bg = cb.BlendGraph(lw, chunks, store, recompute_ratio=0.15, check_layer=1)
    before = bg(chunks, store).clone()
    victim = chunks[2]
    e = store.get(victim.chunk_id)
    K = [k * 1.5 for k in e["K"]]
    V = [v * -1.0 for v in e["V"]]
    store._cache.pop(victim.chunk_id)                 # evicted ...
    store.put(victim.chunk_id, K, V)                  # ... and stored again, other values
    ref, ref_idx = _eager(cb, lw, chunks, store)
    got = bg(chunks, store)
    torch.cuda.synchronize()
    assert torch.equal(got, ref) and torch.equal(bg.idx, ref_idx)
    assert not torch.equal(got, before)


def test_graph_with_kv_arena_slab_reuse():
    """KVArena: a chunk evicted and another stored in its slab (same addresses,
    new values); the replay reads the new values, like the eager path."""
    cb, lw, model, chunks, _ = _setup(CFG_D128, n_chunks=6, chunk_len=300, q_len=40, seed=3)
    kv_dim = model.config.num_key_value_heads * model.config.head_dim
    arena = cb.KVArena(lw.num_layers, kv_dim, sum(c.length for c in chunks) + 300, lw.device)
    for c in chunks:
        cb.precompute_chunk_kv_into(lw, c, arena)
    bg = cb.BlendGraph(lw, chunks, arena, recompute_ratio=0.15, check_layer=1)
    ref0, _ = _eager(cb, lw, chunks, arena)
    assert torch.equal(bg(chunks, arena), ref0)
    # replace chunk 1 by a same-length chunk with other ids: LRU eviction frees its slab
    g = torch.Generator().manual_seed(99)
    t = torch.randint(0, model.config.vocab_size, (chunks[1].length,), generator=g).tolist()
    nc = cb.Chunk(text="swap", token_ids=t, chunk_id=cb.chunker._stable_id("swap", t))
    arena._drop(chunks[1].chunk_id)
    cb.precompute_chunk_kv_into(lw, nc, arena)
    reqs = [chunks[0], nc] + chunks[2:]
    ref, ref_idx = _eager(cb, lw, reqs, arena)
    got = bg(reqs, arena)
    torch.cuda.synchronize()
    assert torch.equal(got, ref) and torch.equal(bg.idx, ref_idx)


@pytest.mark.parametrize("rows", ["all", "last"])
def test_fuse_selective_graph_default_matches_eager(rows):
    cb, lw, model, chunks, store = _setup(CFG_D128, n_chunks=6, chunk_len=300, q_len=40, seed=3)
    other = _other_chunks(cb, lw, chunks, store, 5)
    st = torch.zeros(1, dtype=torch.int32, device="cuda:0")
    outs = []
    for reqs in (chunks, other, chunks, other):
        ref, ref_idx = _eager(cb, lw, reqs, store, logits_rows=rows)
        got, idx = cb.fuse_selective(lw, reqs, store, recompute_ratio=0.15, check_layer=1,
                                     return_hkvd_indices=True, logits_rows=rows, status=st)
        torch.cuda.synchronize()
        assert torch.equal(got, ref) and torch.equal(idx, ref_idx)
        outs.append((got, ref))
    assert int(st.item()) == 0
    for got, ref in outs:                     # earlier results were not overwritten by later calls
        assert torch.equal(got, ref)
    assert len(lw._cbk_graphs) == 1           # one geometry, one graph
    cb.fusor.release_graphs(lw)
    assert len(lw._cbk_graphs) == 0


def test_last_row_logits_equal_dense_last_row():
    cb, lw, model, chunks, store = _setup(CFG_D128, n_chunks=6, chunk_len=300, q_len=40, seed=3)
    dense = cb.fuse_selective(lw, chunks, store, cuda_graph=False)
    last = cb.fuse_selective(lw, chunks, store, cuda_graph=False, logits_rows="last")
    assert last.shape == (1, 1, model.config.vocab_size)
    assert torch.equal(last[0, 0], dense[0, -1])
    out = cb.fuse_selective(lw, chunks, store, logits_rows="last", return_layerwise_output=True)
    assert torch.equal(out.logits[0, 0], dense[0, -1])
    assert out.past_key_values.get_seq_length() == dense.shape[1]
    with pytest.raises(ValueError):
        cb.fuse_selective(lw, chunks, store, logits_rows="some")


def test_layerwise_output_of_replayed_graph_is_owned():
    """The cache fuse_selective returns from a replayed graph is a copy: a later
    call with other chunks does not change it."""
    cb, lw, model, chunks, store = _setup(CFG_D128, n_chunks=6, chunk_len=300, q_len=40, seed=3)
    ref = cb.fuse_selective(lw, chunks, store, return_layerwise_output=True, cuda_graph=False)
    a = cb.fuse_selective(lw, chunks, store, return_layerwise_output=True)
    b = cb.fuse_selective(lw, _other_chunks(cb, lw, chunks, store, 8), store, return_layerwise_output=True)
    torch.cuda.synchronize()
    for l in range(lw.num_layers):
        assert torch.equal(a.past_key_values.layers[l].keys, ref.past_key_values.layers[l].keys)
        assert torch.equal(a.past_key_values.layers[l].values, ref.past_key_values.layers[l].values)
    assert not torch.equal(a.logits, b.logits)
