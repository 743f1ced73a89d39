"""BlendGraph (fuse_selective captured as one CUDA graph) gives the eager
path's logits and selection bit for bit, also for other chunks of the same
lengths after the chunk table and ids are refreshed."""
import pytest
import torch

from test_gpu_fusor import _setup

pytestmark = pytest.mark.gpu


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


@pytest.mark.parametrize("cfg", [None, dict(vocab_size=2000, hidden_size=1024, intermediate_size=2048,
                                            num_hidden_layers=4, num_attention_heads=8, num_key_value_heads=2,
                                            head_dim=128, rope_theta=1e6, rms_norm_eps=1e-5,
                                            max_position_embeddings=8192, sliding_window=None)])
def test_blend_graph_matches_eager(cfg):
    if cfg is None:
        cb, lw, model, chunks, store = _setup()
    else:
        cb, lw, model, chunks, store = _setup(cfg, n_chunks=6, chunk_len=300, q_len=40, seed=3)
    bg = cb.BlendGraph(lw, chunks, store, recompute_ratio=0.15, check_layer=1)
    for reqs in (chunks, _other_chunks(cb, lw, chunks, store, 11), chunks):
        ref, ref_idx = cb.fuse_selective(lw, reqs, store, recompute_ratio=0.15, check_layer=1,
                                         return_hkvd_indices=True)
        got = bg(reqs, store)
        torch.cuda.synchronize()
        assert torch.equal(bg.idx, ref_idx)
        assert torch.equal(got, ref)
    with pytest.raises(ValueError):
        bg(chunks[:-1], store)
