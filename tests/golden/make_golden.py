"""Generate the golden fixtures in this folder from the REFERENCE implementation.

Runs only where the reference sources are available; the fixtures it writes
are committed so that tests on other machines never need the reference.
Usage (the reference checkout's root, the folder holding ``src/cacheblend``,
given by argument or by the CACHEBLEND_REFERENCE environment variable)::

    python tests/golden/make_golden.py --reference <path to cacheblend-hf-v7>

The reference (cacheblend-hf-v7, ``src/cacheblend``) pins transformers 4.49; this
image has 5.5.  Three API breaks are bridged here by monkeypatching transformers
from the outside (no reference file is modified):

1. ``MistralModel._update_causal_mask`` no longer exists.  It is restored as a
   function returning ``None`` (the 4.49 SDPA behaviour), so ``fusor.py:300-307``
   builds its own additive -inf mask and ``forward_layerwise`` runs SDPA with
   ``is_causal``.
2. The decoder-layer kwarg ``past_key_value`` became ``past_key_values``; the
   patched layer forward renames it.
3. Decoder layers return a Tensor instead of a tuple (``model.py:162`` indexes
   ``out[0]``); the patched forward returns a 1-tuple.

Fixtures written:

* ``mock_fp32.npz``   -- the CPU-mock config end to end (fp32): chunk token ids,
  per-chunk pre-RoPE K / V at every layer (``precompute_chunk_kv``), the
  check-layer deviations and selected indices, the fused cache K / V of every
  layer, the selective logits rows, and the full-recompute / full-reuse logits
  of the last position.
* ``kernels_bf16.npz`` -- function-level vectors in bf16 (stored as uint16 bit
  patterns): ``apply_rope_shift``, ``kv_deviation``, ``select_top_k`` (incl.
  ties), the force-include rule of ``fusor.py:344-353`` and the masked SDPA of
  ``fusor.py:385-395``.
"""
from __future__ import annotations

import argparse
import hashlib
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

# CPU-mock configuration (tiny Mistral-style decoder).
MOCK = dict(
    vocab_size=1000, hidden_size=256, intermediate_size=512,
    num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2,
    head_dim=64, rope_theta=1e6, rms_norm_eps=1e-5,
    max_position_embeddings=4096, sliding_window=None,
)
N_CHUNKS, CHUNK_LEN, QUERY_LEN = 4, 128, 32
RATIO, CHECK_LAYER = 0.15, 1


def install_compat_shim():
    """Bridge transformers 5.5 to the 4.49 API the reference calls."""
    from transformers.models.mistral import modeling_mistral as mm
    from transformers.models.llama import modeling_llama as ml

    def _update_causal_mask(self, *args, **kwargs):
        return None

    for mod, model_cls, layer_cls in ((mm, mm.MistralModel, mm.MistralDecoderLayer),
                                      (ml, ml.LlamaModel, ml.LlamaDecoderLayer)):
        model_cls._update_causal_mask = _update_causal_mask
        orig = layer_cls.forward

        def fwd(self, *args, _orig=orig, **kwargs):
            if "past_key_value" in kwargs:
                kwargs["past_key_values"] = kwargs.pop("past_key_value")
            kwargs.pop("cache_position", None)
            out = _orig(self, *args, **kwargs)
            return out if isinstance(out, tuple) else (out,)

        layer_cls.forward = fwd


def build_mock_model(dtype=torch.float32):
    from transformers import MistralConfig, MistralForCausalLM
    torch.manual_seed(0)
    cfg = MistralConfig(**MOCK)
    cfg._attn_implementation = "sdpa"
    model = MistralForCausalLM(cfg).to(dtype).eval()
    return model


def weights_digest(model) -> str:
    h = hashlib.sha256()
    for name, p in sorted(model.state_dict().items()):
        h.update(name.encode())
        h.update(p.detach().float().contiguous().numpy().tobytes())
    return h.hexdigest()


def wrap_layerwise(model):
    """Construct the reference LayerwiseModel the way runners.py:198-215 does."""
    from cacheblend import LayerwiseModel
    lw = LayerwiseModel.__new__(LayerwiseModel)
    lw.model = model
    lw.tokenizer = None
    lw.device = torch.device("cpu")
    lw.dtype = next(model.parameters()).dtype
    lw._inner = model.model
    lw.num_layers = len(lw._inner.layers)
    lw._pre_rope_k = {}
    lw._hook_handles = []
    lw._install_k_proj_hooks()
    return lw


def mock_token_chunks():
    g = torch.Generator().manual_seed(0)
    lens = [CHUNK_LEN] * N_CHUNKS + [QUERY_LEN]
    return [torch.randint(0, MOCK["vocab_size"], (n,), generator=g).tolist() for n in lens]


def make_mock(out_path):
    from cacheblend import KVStore, precompute_chunk_kv
    from cacheblend.chunker import Chunk, _stable_id
    from cacheblend.fusor import fuse_selective, fuse_full_recompute, fuse_full_reuse
    from cacheblend.hkvd import kv_deviation

    model = build_mock_model()
    lw = wrap_layerwise(model)
    chunks = [Chunk(text=f"c{i}", token_ids=ids, chunk_id=_stable_id(f"c{i}", ids))
              for i, ids in enumerate(mock_token_chunks())]
    store = KVStore()
    data = {}
    for ci, c in enumerate(chunks):
        K, V = precompute_chunk_kv(lw, c)
        store.put(c.chunk_id, K, V)
        data[f"ids_{ci}"] = np.asarray(c.token_ids, np.int64)
        for li in range(lw.num_layers):
            data[f"chunkK_{ci}_{li}"] = K[li][0].numpy()
            data[f"chunkV_{ci}_{li}"] = V[li][0].numpy()

    out, idx = fuse_selective(lw, chunks, store, recompute_ratio=RATIO, check_layer=CHECK_LAYER,
                              return_layerwise_output=True, return_hkvd_indices=True)
    S = out.logits.shape[1]
    data["top_indices"] = idx.numpy()
    data["logits_sel"] = out.logits[0, idx].numpy()
    for li in range(lw.num_layers):
        layer = out.past_key_values.layers[li]
        data[f"cacheK_{li}"] = layer.keys[0].numpy()     # (Hkv, S, D)
        data[f"cacheV_{li}"] = layer.values[0].numpy()
    # Deviations exactly as fusor.py:339 computes them (pre-RoPE fresh K vs cached K).
    kfresh = lw.get_pre_rope_k(CHECK_LAYER)
    kcached = torch.cat([store.get(c.chunk_id)["K"][CHECK_LAYER] for c in chunks], dim=1)
    data["kfresh_ck"] = kfresh[0].numpy()
    data["deviations"] = kv_deviation(kfresh, kcached).numpy()

    full = fuse_full_recompute(lw, chunks)
    data["logits_full_last"] = full[0, -1].numpy()
    sel_r1 = fuse_selective(lw, chunks, store, recompute_ratio=1.0)
    data["ratio1_maxdiff"] = np.float32((sel_r1 - full).abs().max().item())
    reuse = fuse_full_reuse(lw, chunks, store)
    data["logits_reuse_last"] = reuse[0, -1].numpy()
    data["weights_sha256"] = np.frombuffer(weights_digest(model).encode(), np.uint8)
    data["S"] = np.int64(S)
    np.savez_compressed(out_path, **data)
    print(f"wrote {out_path}: S={S} k={idx.numel()} last_in={int(idx[-1]) == S - 1}")


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def make_kernels(out_path):
    from transformers import MistralConfig
    from transformers.models.mistral.modeling_mistral import MistralRotaryEmbedding
    from cacheblend.rope import apply_rope_shift
    from cacheblend.hkvd import kv_deviation, select_top_k
    from torch.nn.functional import scaled_dot_product_attention as sdpa

    data = {}
    g = torch.Generator().manual_seed(1)

    # apply_rope_shift in bf16 at Mistral-like head geometry (Hkv=2, D=128), positions up to 40k.
    class _Attn:  # minimal LayerwiseModel stand-in: rope.py:35-40 reads these fields only
        pass
    for name, theta, hkv, d, n in (("mistral", 1e6, 2, 128, 96), ("llama3", 5e5, 2, 128, 64),
                                   ("mock", 1e6, 2, 64, 40)):
        cfg = MistralConfig(hidden_size=hkv * d * 2, num_attention_heads=hkv * 2, num_key_value_heads=hkv,
                            head_dim=d, rope_theta=theta, max_position_embeddings=65536)
        rot = MistralRotaryEmbedding(cfg)
        lw = _Attn()
        lw._inner = _Attn()
        lw._inner.rotary_emb = rot
        lay = _Attn(); lay.self_attn = _Attn(); lay.self_attn.config = cfg; lay.self_attn.head_dim = d
        lw._inner.layers = [lay]
        K = (torch.randn((1, n, hkv * d), generator=g) * 2.0).to(torch.bfloat16)
        pos = torch.randint(0, 40000, (1, n), generator=g)
        pos[0, :4] = torch.tensor([0, 1, 4095, 32767])
        out = apply_rope_shift(K, pos, lw)
        data[f"rope_{name}_K"] = bf16_bits(K[0])
        data[f"rope_{name}_pos"] = pos[0].numpy()
        data[f"rope_{name}_out"] = bf16_bits(out[0])
        data[f"rope_{name}_invfreq"] = rot.inv_freq.numpy()
        data[f"rope_{name}_theta"] = np.float64(theta)

    # kv_deviation on bf16 inputs (hkvd.py:23-55).
    S, F = 300, 256
    Kold = torch.randn((1, S, F), generator=g).to(torch.bfloat16)
    noise = torch.randn((1, S, F), generator=g) * 0.05
    mask = (torch.rand((1, S, 1), generator=g) < 0.2).float()
    Knew = (Kold.float() + noise * mask + 0.001 * torch.randn((1, S, F), generator=g)).to(torch.bfloat16)
    Knew[0, :10] = Kold[0, :10]       # exact zeros (identical prefix rows)
    dev = kv_deviation(Knew, Kold)
    data["dev_Knew"] = bf16_bits(Knew[0])
    data["dev_Kold"] = bf16_bits(Kold[0])
    data["dev_out"] = dev.numpy()
    for r in (0.001, 0.1, 0.15, 0.5, 0.999, 1.0):
        data[f"topk_{r}"] = select_top_k(dev, r).numpy()

    # select_top_k with distinct random values of several sizes (tie-free boundary).
    for n in (1, 7, 544, 6208):
        v = torch.rand((n,), generator=g)
        data[f"topk_rand_{n}"] = v.numpy()
        data[f"topk_rand_{n}_idx"] = select_top_k(v, 0.15).numpy()

    # Force-include rule (fusor.py:344-353) on a case where the last position is not selected.
    v = torch.rand((200,), generator=g)
    v[-1] = -1.0
    idx = select_top_k(v, 0.15)
    last = 199
    if last not in idx.tolist():
        sel = v[idx]
        drop = idx[sel.argmin()].item()
        idx = torch.tensor(sorted([i for i in idx.tolist() if i != drop] + [last]))
    data["force_dev"] = v.numpy()
    data["force_idx"] = idx.numpy()

    # Masked partial-query SDPA (fusor.py:381-399) in bf16: GQA n_rep=2, causal by position.
    Hq, Hkv, D, S2 = 4, 2, 64, 160
    sel = torch.sort(torch.randperm(S2, generator=g)[:24]).values
    sel[-1] = S2 - 1
    sel = torch.sort(torch.unique(sel)).values
    q = torch.randn((1, Hq, sel.numel(), D), generator=g).to(torch.bfloat16)
    k = torch.randn((1, Hkv, S2, D), generator=g).to(torch.bfloat16)
    vv = torch.randn((1, Hkv, S2, D), generator=g).to(torch.bfloat16)
    mask = torch.zeros((1, 1, S2, S2), dtype=torch.bfloat16)
    mask.masked_fill_(torch.triu(torch.ones(S2, S2, dtype=torch.bool), diagonal=1), float("-inf"))
    o = sdpa(q, k.repeat_interleave(2, dim=1), vv.repeat_interleave(2, dim=1),
             attn_mask=mask[:, :, sel, :S2], scale=D ** -0.5)
    data["attn_q"] = bf16_bits(q[0])
    data["attn_k"] = bf16_bits(k[0])
    data["attn_v"] = bf16_bits(vv[0])
    data["attn_pos"] = sel.numpy()
    data["attn_out"] = bf16_bits(o[0])
    np.savez_compressed(out_path, **data)
    print(f"wrote {out_path}")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("CACHEBLEND_REFERENCE"),
                    help="root of the cacheblend-hf-v7 checkout (default: $CACHEBLEND_REFERENCE)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference or set CACHEBLEND_REFERENCE to the reference checkout")
    sys.path.insert(0, os.path.join(args.reference, "src"))
    torch.set_num_threads(1)           # fixed CPU reduction order for reproducible fixtures
    install_compat_shim()
    make_mock(os.path.join(HERE, "mock_fp32.npz"))
    make_kernels(os.path.join(HERE, "kernels_bf16.npz"))


if __name__ == "__main__":
    main()
