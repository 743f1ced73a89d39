"""End-to-end fuse_selective on the GPU against the oracle.

The device run selects its indices from its own bf16 check-layer K; the oracle
re-derives that selection bit for bit from the same inputs (deviation order is
fixed), and then replays the whole selective forward in fp32 with the same
selection.  Logits are held to the reference's Tolerance.MIXED_SHAPE bound
(max |diff| < 5e-2) at the selected rows and the decode argmax at the last
position must agree; the fused cache is bit-exact where it is pure data
movement (cached V, RoPE of cached K given the device cos/sin table)."""
import numpy as np
import pytest
import torch

from helpers import golden, mock_model, to_bits
from oracle import hotpath as hp, model as om
from oracle.bf16 import bf16_to_f32, f32_to_bf16

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _setup(cfg_kwargs=None, n_chunks=4, chunk_len=128, q_len=32, seed=0):
    import cacheblend as cb
    if cfg_kwargs is None:
        model = mock_model(torch.bfloat16, DEV).eval()
        g = golden("mock_fp32.npz")
        ids = [g[f"ids_{i}"].tolist() for i in range(5)]
    else:
        from transformers import MistralConfig, MistralForCausalLM
        torch.manual_seed(seed)
        cfg = MistralConfig(**cfg_kwargs)
        cfg._attn_implementation = "sdpa"
        model = MistralForCausalLM(cfg).to(torch.bfloat16).to(DEV).eval()
        gen = torch.Generator().manual_seed(seed)
        lens = [chunk_len] * n_chunks + [q_len]
        ids = [torch.randint(0, cfg.vocab_size, (n,), generator=gen).tolist() for n in lens]
    lw = cb.LayerwiseModel.from_hf(model)
    chunks = [cb.Chunk(text=f"c{i}", token_ids=t, chunk_id=cb.chunker._stable_id(f"c{i}", t))
              for i, t in enumerate(ids)]
    store = cb.KVStore()
    for c in chunks:
        K, V = cb.precompute_chunk_kv(lw, c)
        store.put(c.chunk_id, K, V)
    return cb, lw, model, chunks, store


def _oracle_weights(model):
    cfg = om.Config.from_hf(model.config)
    sd = {n: t.float().cpu().numpy() for n, t in model.state_dict().items()}
    return om.Weights(sd, cfg, model.model.rotary_emb.inv_freq.float().cpu().numpy())


def _check_selective(cb, lw, model, chunks, store, ratio=0.15, ck=1):
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    out, idx = cb.fuse_selective(lw, chunks, store, recompute_ratio=ratio, check_layer=ck,
                                 return_layerwise_output=True, return_hkvd_indices=True, status=st)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    S = sum(c.length for c in chunks)
    k = max(1, min(S, int(S * ratio)))
    idx_np = idx.cpu().numpy()
    assert idx.dtype == torch.int64 and idx_np.shape == (k,)
    assert np.all(np.diff(idx_np) > 0) and idx_np[-1] == S - 1
    assert out.logits.shape == (1, S, model.config.vocab_size)

    entries = [store.get(c.chunk_id) for c in chunks]
    L = lw.num_layers
    # (c) the selection, re-derived by the oracle from the device's own check-layer K
    k_fresh = to_bits(lw.get_pre_rope_k(ck)[0])
    k_cached = np.concatenate([to_bits(e["K"][ck][0]) for e in entries])
    dev = hp.kv_deviation(bf16_to_f32(k_fresh), bf16_to_f32(k_cached))
    np.testing.assert_array_equal(idx_np, hp.topk_select(dev, k, force_last=True))

    # (a)+(b)+(d) the fused cache of every cached layer
    rot = model.model.rotary_emb
    tab = cb.ops.rope_table(rot.inv_freq, S).cpu().numpy()
    invf = rot.inv_freq.float().cpu().numpy()
    attn0 = model.model.layers[0].self_attn
    D, Hkv = attn0.head_dim, model.config.num_key_value_heads
    rest = np.setdiff1d(np.arange(S), idx_np)
    cache = out.past_key_values
    assert len(cache.layers) == L
    for l in range(L):
        kl, vl = cache.layers[l].keys, cache.layers[l].values
        assert kl.shape == (1, Hkv, S, D) and vl.shape == (1, Hkv, S, D)
        if l < ck:
            continue
        got_k = to_bits(kl[0].permute(1, 0, 2).reshape(S, -1))
        got_v = to_bits(vl[0].permute(1, 0, 2).reshape(S, -1))
        cat_k = np.concatenate([to_bits(e["K"][l][0]) for e in entries])
        cat_v = np.concatenate([to_bits(e["V"][l][0]) for e in entries])
        exp_k = f32_to_bf16(hp.apply_rope(cat_k, np.arange(S), invf, D, "bf16", "ref", cos_sin=tab))
        np.testing.assert_array_equal(got_k[rest], exp_k[rest])
        np.testing.assert_array_equal(got_v[rest], cat_v[rest])
        if l == ck:   # fresh rows of the check layer: RoPE(full-forward K) at their positions
            exp_f = f32_to_bf16(hp.apply_rope(k_fresh[idx_np], idx_np, invf, D, "bf16", "ref", cos_sin=tab))
            np.testing.assert_array_equal(got_k[idx_np], exp_f)

    # whole forward: oracle fp32 replay with the device's selection and chunk KV
    W = _oracle_weights(model)
    ids = [np.asarray(c.token_ids) for c in chunks]
    ck_k = [[bf16_to_f32(to_bits(e["K"][l][0])) for l in range(L)] for e in entries]
    ck_v = [[bf16_to_f32(to_bits(e["V"][l][0])) for l in range(L)] for e in entries]
    r = om.fuse_selective(ids, ck_k, ck_v, W, ratio, ck, force_idx=idx_np)
    got = out.logits[0].float().cpu().numpy()
    diff = np.abs(got[idx_np] - r.logits[idx_np])
    assert diff.max() < 5e-2, diff.max()
    assert np.all(got[rest] == 0)
    assert int(np.argmax(got[-1])) == int(np.argmax(r.logits[-1]))
    return out, idx


def test_fuse_selective_mock_config():
    cb, lw, model, chunks, store = _setup()
    _check_selective(cb, lw, model, chunks, store)
    # the pre-RoPE K hooks fire like the reference's: full rows up to the check
    # layer, selected rows after it
    assert lw.get_pre_rope_k(0).shape[1] == 544 and lw.get_pre_rope_k(1).shape[1] == 544
    assert lw.get_pre_rope_k(1).shape[0] == 1


def test_fuse_selective_head_dim_128_gqa4():
    cfg = dict(vocab_size=2000, hidden_size=1024, intermediate_size=2048, num_hidden_layers=4,
               num_attention_heads=8, num_key_value_heads=2, head_dim=128, rope_theta=1e6,
               rms_norm_eps=1e-5, max_position_embeddings=8192, sliding_window=None)
    cb, lw, model, chunks, store = _setup(cfg, n_chunks=6, chunk_len=300, q_len=40, seed=3)
    _check_selective(cb, lw, model, chunks, store, ratio=0.2, ck=2)


def test_shortcuts_and_errors():
    cb, lw, model, chunks, store = _setup()
    full = cb.fuse_full_recompute(lw, chunks)
    # ratio >= 1 and single chunk are the full-recompute path itself (IDENTICAL_PATH)
    cb.assert_logits_close(cb.fuse_selective(lw, chunks, store, recompute_ratio=1.0), full,
                           cb.Tolerance.IDENTICAL_PATH)
    one = cb.fuse_selective(lw, chunks[:1], store, recompute_ratio=0.15)
    cb.assert_logits_close(one, cb.fuse_full_recompute(lw, chunks[:1]), cb.Tolerance.IDENTICAL_PATH)
    reuse = cb.fuse_selective(lw, chunks, store, recompute_ratio=0.0)
    assert reuse.shape == full.shape
    missing = cb.Chunk(text="x", token_ids=[1, 2, 3], chunk_id="nope")
    with pytest.raises(KeyError):
        cb.fuse_selective(lw, chunks + [missing], store)
    with pytest.raises(IndexError):
        cb.fuse_selective(lw, chunks, store, check_layer=5)


def test_decode_continues_from_blended_cache():
    """The returned cache drives HF decode like the reference's DynamicCache."""
    cb, lw, model, chunks, store = _setup()
    out = cb.fuse_selective(lw, chunks, store, return_layerwise_output=True)
    nxt = out.logits[0, -1].argmax().view(1, 1)
    with torch.inference_mode():
        step = model(input_ids=nxt, past_key_values=out.past_key_values, use_cache=True)
    assert step.logits.shape == (1, 1, model.config.vocab_size)
    assert step.past_key_values.get_seq_length() == 545
    assert torch.isfinite(step.logits).all()


def test_apply_rope_shift_api():
    cb, lw, model, chunks, store = _setup()
    k = golden("kernels_bf16.npz")
    e = store.get(chunks[1].chunk_id)
    K = e["K"][1]                                   # (1, 128, Hkv*D) pre-RoPE
    pos = torch.arange(128, 256, device=DEV).unsqueeze(0)
    out = cb.apply_rope_shift(K, pos, lw)
    assert out.shape == K.shape and out.dtype == K.dtype
    D = model.model.layers[0].self_attn.head_dim
    exp = hp.apply_rope(to_bits(K[0]), np.arange(128, 256), model.model.rotary_emb.inv_freq.float().cpu().numpy(),
                        D, "bf16", "ref")
    from helpers import ulp_diff_bf16
    ud = ulp_diff_bf16(to_bits(out[0]), f32_to_bf16(exp))
    assert ud.max() <= 1 and (ud == 0).mean() > 0.999
    del k
