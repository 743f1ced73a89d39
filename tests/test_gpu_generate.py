"""Greedy decode over the blended cache on the libcbk kernels against the
reference's decode (HF forward with past_key_values = the blended
DynamicCache, runners.py:106-152), fed the same tokens: every step's logits
within the reference's Tolerance.MIXED_SHAPE bound (5e-2), and the same
greedy choice wherever HF's top-2 gap is wider than that bound."""
import pytest
import torch

from test_gpu_fusor import _setup

pytestmark = pytest.mark.gpu


def _compare(cb, lw, model, chunks, store, n_new, ratio=0.15, ck=1):
    tokens, rows = cb.generate_greedy(lw, chunks, store, n_new, recompute_ratio=ratio, check_layer=ck,
                                      return_logits=True)
    assert len(tokens) == n_new == len(rows)
    with torch.inference_mode():
        out = cb.fuse_selective(lw, chunks, store, recompute_ratio=ratio, check_layer=ck,
                                return_layerwise_output=True)
        cache = out.past_key_values
        ref_rows = [out.logits[0, -1]]
        for t in tokens[:-1]:
            step = model(input_ids=torch.tensor([[t]], device=lw.device), past_key_values=cache, use_cache=True)
            cache = step.past_key_values
            ref_rows.append(step.logits[0, -1])
    assert torch.equal(rows[0], ref_rows[0])                  # token 1: the same prefill row
    for i, (ours, ref) in enumerate(zip(rows, ref_rows)):
        diff = (ours.float() - ref.float()).abs().max().item()
        assert diff < 5e-2, (i, diff)
        top2 = torch.topk(ref.float(), 2).values
        if (top2[0] - top2[1]).item() > 5e-2:
            assert tokens[i] == int(ref.argmax())
    return tokens


def test_decode_mock_config():
    cb, lw, model, chunks, store = _setup()
    _compare(cb, lw, model, chunks, store, 8)


def test_decode_head_dim_128_gqa4():
    cfg = dict(vocab_size=2000, hidden_size=1024, intermediate_size=2048, num_hidden_layers=4,
               num_attention_heads=8, num_key_value_heads=2, head_dim=128, rope_theta=1e6,
               rms_norm_eps=1e-5, max_position_embeddings=8192, sliding_window=None)
    cb, lw, model, chunks, store = _setup(cfg, n_chunks=6, chunk_len=300, q_len=40, seed=3)
    _compare(cb, lw, model, chunks, store, 6, ratio=0.2, ck=2)


def test_decode_shortcut_path_and_eos():
    cb, lw, model, chunks, store = _setup()
    toks = cb.generate_greedy(lw, chunks, store, 4, recompute_ratio=1.0)       # reference path
    assert len(toks) == 4
    first = cb.generate_greedy(lw, chunks, store, 1)
    stopped = cb.generate_greedy(lw, chunks, store, 5, eos_token_id=first[0])
    assert stopped == first                                                    # eos right away
    assert cb.generate_greedy(lw, chunks, store, 0) == []


def test_decode_graph_replay_equals_eager():
    """The decode step captured once and replayed gives the eager loop's tokens
    and logits bit for bit (same kernels, same buffers)."""
    cb, lw, model, chunks, store = _setup()
    t1, r1 = cb.generate_greedy(lw, chunks, store, 7, return_logits=True, use_graph=True)
    t2, r2 = cb.generate_greedy(lw, chunks, store, 7, return_logits=True, use_graph=False)
    assert t1 == t2
    for a, b in zip(r1, r2):
        assert torch.equal(a, b)
