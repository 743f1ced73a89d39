"""Pin the oracle against golden vectors produced by the reference itself
(tests/golden/make_golden.py).  CPU only."""
import numpy as np
import pytest
import torch

from helpers import golden, mock_model
from oracle import hotpath as hp, model as om
from oracle.bf16 import bf16_to_f32, f32_to_bf16


@pytest.fixture(scope="module")
def g():
    return golden("mock_fp32.npz")


@pytest.fixture(scope="module")
def k():
    return golden("kernels_bf16.npz")


@pytest.fixture(scope="module")
def weights():
    m = mock_model()
    cfg = om.Config.from_hf(m.config)
    return om.Weights({n: t.numpy() for n, t in m.state_dict().items()}, cfg,
                      m.model.rotary_emb.inv_freq.numpy())


def _chunks(g):
    ids = [g[f"ids_{i}"] for i in range(5)]
    K = [[g[f"chunkK_{i}_{l}"] for l in range(2)] for i in range(5)]
    V = [[g[f"chunkV_{i}_{l}"] for l in range(2)] for i in range(5)]
    return ids, K, V


def test_mock_weights_match_fixture(g):
    from golden.make_golden import weights_digest
    assert weights_digest(mock_model()) == bytes(g["weights_sha256"]).decode()


def test_precompute_chunk_kv_matches_reference(g, weights):
    ids, K, V = _chunks(g)
    for i in range(5):
        k_o, v_o = om.precompute_chunk_kv(ids[i], weights)
        for l in range(2):
            np.testing.assert_allclose(k_o[l], K[i][l], atol=5e-6, rtol=0)
            np.testing.assert_allclose(v_o[l], V[i][l], atol=5e-6, rtol=0)


def test_fuse_selective_matches_reference(g, weights):
    ids, K, V = _chunks(g)
    r = om.fuse_selective(ids, K, V, weights, 0.15, 1)
    assert int(g["S"]) == 544 and len(r.indices) == 81 == hp.topk_count(544, 0.15)
    np.testing.assert_array_equal(r.indices, g["top_indices"])
    assert r.indices[-1] == 543                          # last position always selected
    assert np.all(np.diff(r.indices) > 0)                # ascending
    # deviations: fixed kernel order vs torch's order -> rounding-level differences
    np.testing.assert_allclose(r.deviations, g["deviations"], rtol=1e-5, atol=1e-9)
    # logits at the selected rows: Tolerance.SAME_SHAPE (< 1e-3) of the reference
    assert np.abs(r.logits[r.indices] - g["logits_sel"]).max() < 1e-4
    assert np.all(r.logits[np.setdiff1d(np.arange(544), r.indices)] == 0)
    for l in range(2):
        ref_k = g[f"cacheK_{l}"].transpose(1, 0, 2).reshape(544, -1)
        ref_v = g[f"cacheV_{l}"].transpose(1, 0, 2).reshape(544, -1)
        assert np.abs(r.cache_k[l] - ref_k).max() < 1e-5
        assert np.abs(r.cache_v[l] - ref_v).max() < 1e-5


def test_full_recompute_matches_reference(g, weights):
    ids, _, _ = _chunks(g)
    logits, _ = om.forward_full(np.concatenate(ids), weights)
    assert np.abs(logits[-1] - g["logits_full_last"]).max() < 1e-4
    assert float(g["ratio1_maxdiff"]) == 0.0     # reference: ratio=1 shortcut is IDENTICAL_PATH


@pytest.mark.parametrize("name,head_dim", [("mistral", 128), ("llama3", 128), ("mock", 64)])
def test_rope_ref_mode_bit_exact(k, name, head_dim):
    """HF apply_rotary_pos_emb in bf16 (reference rope.py:33-64) reproduced bit for bit."""
    out = hp.apply_rope(k[f"rope_{name}_K"], k[f"rope_{name}_pos"], k[f"rope_{name}_invfreq"],
                        head_dim, "bf16", "ref")
    np.testing.assert_array_equal(f32_to_bf16(out), k[f"rope_{name}_out"])


@pytest.mark.parametrize("name,head_dim", [("mistral", 128), ("llama3", 128)])
def test_rope_fp32_mode_closer_to_exact(k, name, head_dim):
    x = bf16_to_f32(k[f"rope_{name}_K"])
    pos, invf = k[f"rope_{name}_pos"], k[f"rope_{name}_invfreq"]
    exact = hp.apply_rope_f64(x, pos, invf, head_dim)
    err_fp32 = np.abs(hp.apply_rope(x, pos, invf, head_dim, "bf16", "fp32") - exact).mean()
    err_ref = np.abs(bf16_to_f32(k[f"rope_{name}_out"]) - exact).mean()
    assert err_fp32 < err_ref


def test_inv_freq_restatement(k):
    for name, d in (("mistral", 128), ("llama3", 128), ("mock", 64)):
        ours = hp.inv_freq(float(k[f"rope_{name}_theta"]), d)
        np.testing.assert_allclose(ours, k[f"rope_{name}_invfreq"], rtol=2e-7)


def test_kv_deviation(k):
    dev = hp.kv_deviation(bf16_to_f32(k["dev_Knew"]), bf16_to_f32(k["dev_Kold"]))
    np.testing.assert_allclose(dev, k["dev_out"], rtol=1e-6, atol=0)
    assert np.all(dev[:10] == 0)          # identical rows -> exactly zero


def test_kv_deviation_errors():
    with pytest.raises(ValueError):
        hp.kv_deviation(np.zeros((4, 8)), np.zeros((4, 16)))
    with pytest.raises(NotImplementedError):
        hp.kv_deviation(np.zeros((2, 4, 8)), np.zeros((2, 4, 8)))
    with pytest.raises(ValueError):
        hp.kv_deviation(np.zeros((8,)), np.zeros((8,)))


@pytest.mark.parametrize("ratio", [0.001, 0.1, 0.15, 0.5, 1.0])
def test_select_top_k_tie_free(k, ratio):
    np.testing.assert_array_equal(hp.select_top_k(k["dev_out"], ratio), k[f"topk_{ratio}"])


def test_select_top_k_ties_documented(k):
    """k=299 of 300 must drop one of ten exact zeros: torch's CPU topk keeps an
    unspecified one; the oracle (and the kernel) keep the lowest indices.  Every
    element above the tie value is selected by both."""
    ours = hp.select_top_k(k["dev_out"], 0.999)
    ref = k["topk_0.999"]
    assert len(ours) == len(ref) == 299
    dev = k["dev_out"]
    above = set(np.nonzero(dev > 0)[0].tolist())
    assert above <= set(ours.tolist()) and above <= set(ref.tolist())
    assert 9 not in set(ours.tolist()) and 0 in set(ours.tolist())


@pytest.mark.parametrize("n", [1, 7, 544, 6208])
def test_select_top_k_random(k, n):
    np.testing.assert_array_equal(hp.select_top_k(k[f"topk_rand_{n}"], 0.15), k[f"topk_rand_{n}_idx"])


def test_force_include(k):
    idx = hp.topk_select(k["force_dev"], hp.topk_count(200, 0.15), force_last=True)
    np.testing.assert_array_equal(idx, k["force_idx"])
    np.testing.assert_array_equal(
        hp.force_include_last(hp.select_top_k(k["force_dev"], 0.15), k["force_dev"]), k["force_idx"])


def test_topk_count_matches_python_int():
    for S in (1, 2, 7, 544, 6208, 32896, 131328):
        for r in (1e-9, 0.001, 0.1, 0.15, 0.3333, 0.5, 0.999, 1.0):
            assert hp.topk_count(S, r) == max(1, min(S, int(S * r)))


def test_partial_attention_matches_reference_sdpa(k):
    q = bf16_to_f32(k["attn_q"]).transpose(1, 0, 2)
    kk = bf16_to_f32(k["attn_k"]).transpose(1, 0, 2)
    v = bf16_to_f32(k["attn_v"]).transpose(1, 0, 2)
    o = hp.partial_attention(q, kk, v, k["attn_pos"], 64 ** -0.5)
    ref = bf16_to_f32(k["attn_out"]).transpose(1, 0, 2).reshape(o.shape)
    assert np.abs(o - ref).max() < 2e-2     # bf16 SDPA vs exact math


def test_concat_and_scatter_bit_exact():
    rng = np.random.default_rng(0)
    parts = [rng.integers(0, 65535, size=(n, 32), dtype=np.uint16) for n in (5, 1, 17)]
    cat = hp.concat_chunks(parts)
    np.testing.assert_array_equal(cat, np.concatenate(parts))
    idx = np.array([0, 6, 22])
    fresh = rng.integers(0, 65535, size=(3, 32), dtype=np.uint16)
    out = hp.scatter_rows(cat, idx, fresh)
    np.testing.assert_array_equal(out[idx], fresh)
    keep = np.setdiff1d(np.arange(23), idx)
    np.testing.assert_array_equal(out[keep], cat[keep])
