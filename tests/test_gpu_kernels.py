"""Kernel-level parity of the sm_100a path against the oracle (and, through the
golden fixtures, against the reference).  Integer / byte work is bit-exact;
RoPE is bit-exact given the device's cos/sin table; attention is compared with
an exact fp64 oracle element by element, within a bound that scales with the
output (``attn_check``)."""
import numpy as np
import pytest
import torch

import attn_check as ac
from helpers import from_bits, golden, to_bits, ulp_diff_bf16
from oracle import hotpath as hp
from oracle.bf16 import bf16_to_f32, f32_to_bf16, f16_to_f32, f32_to_f16

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
DT = {"bf16": torch.bfloat16, "f16": torch.float16}
ENC = {"bf16": f32_to_bf16, "f16": f32_to_f16}
DEC = {"bf16": bf16_to_f32, "f16": f16_to_f32}


@pytest.fixture(scope="module")
def ops():
    from cacheblend import ops as o
    return o


def status_word():
    return torch.zeros(1, dtype=torch.int32, device=DEV)


def assert_status_clean(st):
    torch.cuda.synchronize()
    assert int(st.item()) == 0, f"device status bits {int(st.item())}"


def rand16(shape, dtype, gen, scale=1.0):
    return (torch.randn(shape, generator=gen) * scale).to(DT[dtype])


def invf_for(theta, d):
    return torch.from_numpy(hp.inv_freq(theta, d))


# ---------------------------------------------------------------------------
# RoPE
# ---------------------------------------------------------------------------
def test_rope_table_matches_oracle(ops):
    invf = invf_for(1e6, 128)
    tab = ops.rope_table(invf.to(DEV), 40000).cpu().numpy()
    c, s = hp.rope_cos_sin(invf.numpy(), np.arange(40000))
    assert np.abs(tab[..., 0] - c).max() <= 2.5e-7
    assert np.abs(tab[..., 1] - s).max() <= 2.5e-7


@pytest.mark.parametrize("name,head_dim", [("mistral", 128), ("llama3", 128), ("mock", 64)])
def test_rope_rows_vs_reference_golden(ops, name, head_dim):
    """apply_rope_shift outputs of the reference (bf16): within 1 ulp everywhere
    and bit-exact on >= 99.9% of elements (the fp32 cos/sin of CUDA and of the
    reference's CPU math may differ by an ulp)."""
    k = golden("kernels_bf16.npz")
    x = from_bits(k[f"rope_{name}_K"], device=DEV)
    pos = torch.from_numpy(k[f"rope_{name}_pos"]).to(DEV)
    tab = ops.rope_table(torch.from_numpy(k[f"rope_{name}_invfreq"]).to(DEV), int(pos.max()) + 1)
    st = status_word()
    out = to_bits(ops.rope_rows(x, pos, tab, head_dim, mode="ref", status=st))
    ref = k[f"rope_{name}_out"]
    assert_status_clean(st)
    ud = ulp_diff_bf16(out, ref)
    assert ud.max() <= 1
    assert (ud == 0).mean() >= 0.999


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("mode", ["ref", "fp32"])
def test_rope_rows_bit_exact_given_table(ops, dtype, mode):
    g = torch.Generator().manual_seed(3)
    x = rand16((300, 8 * 128), dtype, g, 3.0)
    pos = torch.randint(0, 131072, (300,), generator=g)
    invf = invf_for(5e5, 128)
    tab = ops.rope_table(invf.to(DEV), 131072)
    out = ops.rope_rows(x.to(DEV), pos.to(DEV), tab, 128, mode=mode).cpu()
    exp = hp.apply_rope(to_bits(x), pos.numpy(), invf.numpy(), 128, dtype, mode,
                        cos_sin=tab.cpu().numpy())
    np.testing.assert_array_equal(to_bits(out), ENC[dtype](exp))


# ---------------------------------------------------------------------------
# (a)+(b) assemble
# ---------------------------------------------------------------------------
def _make_store(lengths, n_layers, kv_dim, dtype, gen):
    entries = []
    for n in lengths:
        entries.append({"K": [rand16((1, n, kv_dim), dtype, gen, 2.0).to(DEV) for _ in range(n_layers)],
                        "V": [rand16((1, n, kv_dim), dtype, gen).to(DEV) for _ in range(n_layers)]})
    return entries


@pytest.mark.parametrize("dtype,n_kv,head_dim,lengths", [
    ("bf16", 8, 128, [1024, 1024, 1024, 1024, 1024, 1024, 64]),
    ("bf16", 2, 64, [128, 128, 128, 128, 32]),
    ("f16", 8, 128, [1, 17, 300, 5]),
    ("bf16", 1, 128, [3]),
])
def test_assemble_kv(ops, dtype, n_kv, head_dim, lengths):
    g = torch.Generator().manual_seed(len(lengths))
    L, lo = 4, 1
    kv_dim = n_kv * head_dim
    entries = _make_store(lengths, L, kv_dim, dtype, g)
    table = ops.ChunkTable(entries, range(lo, L), torch.device(DEV))
    S = sum(lengths)
    invf = invf_for(1e6, head_dim)
    rope = ops.rope_table(invf.to(DEV), S + 5)
    fk = torch.full((L, S, kv_dim), 7.0, dtype=DT[dtype], device=DEV)
    fv = torch.full_like(fk, 7.0)
    st = status_word()
    ops.assemble_kv(table, lo, L, n_kv, head_dim, rope, fk, fv, mode="ref", status=st)
    assert_status_clean(st)
    tab = rope.cpu().numpy()
    for l in range(L):
        if l < lo:       # untouched
            assert torch.all(fk[l] == 7.0) and torch.all(fv[l] == 7.0)
            continue
        cat_k = hp.concat_chunks([to_bits(e["K"][l][0]) for e in entries])
        cat_v = hp.concat_chunks([to_bits(e["V"][l][0]) for e in entries])
        np.testing.assert_array_equal(to_bits(fv[l]), cat_v)
        exp = hp.apply_rope(cat_k, np.arange(S), invf.numpy(), head_dim, dtype, "ref", cos_sin=tab)
        np.testing.assert_array_equal(to_bits(fk[l]), ENC[dtype](exp))


def test_assemble_reports_bad_positions(ops):
    g = torch.Generator().manual_seed(9)
    entries = _make_store([16, 16], 1, 128, "bf16", g)
    table = ops.ChunkTable(entries, [0], torch.device(DEV))
    rope = ops.rope_table(invf_for(1e6, 128).to(DEV), 20)
    pos = torch.arange(32, device=DEV, dtype=torch.int64)      # rows 20..31 beyond the table
    fk = torch.zeros((1, 32, 128), dtype=torch.bfloat16, device=DEV)
    fv = torch.zeros_like(fk)
    st = status_word()
    ops.assemble_kv(table, 0, 1, 1, 128, rope, fk, fv, positions=pos, status=st)
    torch.cuda.synchronize()
    assert int(st.item()) & 1
    assert torch.all(fk[0, 20:] == 0)                          # skipped, not written


# ---------------------------------------------------------------------------
# (b)+(d) fresh rows
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("by_row", [False, True])
@pytest.mark.parametrize("gather", [True, False])
@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("nq,nkv,D,mode", [
    (8, 2, 128, "ref"),      # head_dim 128: the compile-time instance
    (8, 2, 128, "fp32"),
    (3, 1, 128, "ref"),      # Q and K units only partly filled
    (4, 2, 64, "ref"),       # generic instance, D/16 divides 32 (one cos/sin slice per lane)
    (6, 3, 96, "ref"),       # D/16 = 6 does not divide 32: a cos/sin slice per pair group
    (6, 3, 96, "fp32"),
    (2, 1, 256, "ref"),
])
def test_rope_scatter(ops, by_row, gather, dtype, nq, nkv, D, mode):
    """by_row: the cos/sin table holds the selection's rows (row j = position
    idx[j]), as fuse_selective passes it; same bits as the position table."""
    g = torch.Generator().manual_seed(5)
    S = 700
    idx = torch.sort(torch.randperm(S, generator=g)[:105]).values
    n_src = S if gather else idx.numel()
    q = rand16((n_src, nq * D), dtype, g, 2.0).to(DEV)
    k = rand16((n_src, nkv * D), dtype, g, 2.0).to(DEV)
    v = rand16((n_src, nkv * D), dtype, g).to(DEV)
    kc = rand16((S, nkv * D), dtype, g).to(DEV)
    vc = rand16((S, nkv * D), dtype, g).to(DEV)
    kc0, vc0 = to_bits(kc), to_bits(vc)
    invf = invf_for(1e6, D)
    rope = ops.rope_table(invf.to(DEV), S)
    st = status_word()
    tab_arg = rope.index_select(0, idx.to(DEV)) if by_row else rope
    qo = ops.rope_scatter(q, k, v, idx.to(DEV), gather, S, nq, nkv, D, tab_arg, kc, vc, mode=mode, status=st,
                          table_by_row=by_row)
    assert_status_clean(st)
    tab = rope.cpu().numpy()
    rows = idx.numpy() if gather else np.arange(idx.numel())
    pos = idx.numpy()
    exp_q = hp.apply_rope(to_bits(q)[rows], pos, invf.numpy(), D, dtype, mode, cos_sin=tab)
    np.testing.assert_array_equal(to_bits(qo), ENC[dtype](exp_q))
    exp_k = hp.apply_rope(to_bits(k)[rows], pos, invf.numpy(), D, dtype, mode, cos_sin=tab)
    np.testing.assert_array_equal(to_bits(kc), hp.scatter_rows(kc0, pos, ENC[dtype](exp_k)))
    np.testing.assert_array_equal(to_bits(vc), hp.scatter_rows(vc0, pos, to_bits(v)[rows]))


# ---------------------------------------------------------------------------
# (c) HKVD
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("dtype,feat,lengths", [
    ("bf16", 1024, [1024] * 6 + [64]), ("bf16", 128, [128] * 4 + [32]), ("f16", 256, [7, 1, 300]),
    ("bf16", 8, [5, 5]),
])
def test_kv_deviation_bit_exact(ops, dtype, feat, lengths):
    g = torch.Generator().manual_seed(feat)
    entries = _make_store(lengths, 1, feat, dtype, g)
    S = sum(lengths)
    old = torch.cat([e["K"][0][0] for e in entries]).cpu()
    noise = torch.randn((S, feat), generator=g) * 0.05 * (torch.rand((S, 1), generator=g) < 0.2)
    new = (old.float() + noise).to(DT[dtype])
    new[: lengths[0]] = old[: lengths[0]]
    table = ops.ChunkTable(entries, [0], torch.device(DEV))
    dev = ops.kv_deviation_rows(new.to(DEV), table, 0).cpu().numpy()
    exp = hp.kv_deviation(DEC[dtype](to_bits(new)), DEC[dtype](to_bits(old)))
    np.testing.assert_array_equal(dev.view(np.uint32), exp.view(np.uint32))
    assert np.all(dev[: lengths[0]] == 0)


def test_kv_deviation_api_vs_reference_golden():
    from cacheblend import kv_deviation
    k = golden("kernels_bf16.npz")
    new = from_bits(k["dev_Knew"], device=DEV)
    old = from_bits(k["dev_Kold"], device=DEV)
    dev = kv_deviation(new.unsqueeze(0), old.unsqueeze(0)).cpu().numpy()
    np.testing.assert_allclose(dev, k["dev_out"], rtol=1e-6, atol=0)
    exp = hp.kv_deviation(bf16_to_f32(k["dev_Knew"]), bf16_to_f32(k["dev_Kold"]))
    np.testing.assert_array_equal(dev, exp)
    with pytest.raises(ValueError):
        kv_deviation(new, old[:5])
    with pytest.raises(NotImplementedError):
        kv_deviation(new.expand(2, *new.shape), old.expand(2, *old.shape))


def _topk_cases():
    rng = np.random.default_rng(11)
    cases = []
    # sizes at the edges of the kernel's size classes: 8, 16 and 33 keys per thread in
    # registers (S <= 8192, 16384, 33792), keys in shared memory (S <= 40960), keys
    # re-read from global memory
    for S in (1, 2, 7, 544, 1025, 6208, 8192, 8193, 16384, 16385, 33792, 33793, 40960, 40961, 131328):
        cases.append((f"rand{S}", rng.random(S, dtype=np.float32)))
    for S in (9000, 20000):
        q = np.round(rng.random(S) * 16).astype(np.float32)
        q[-1] = 8.0
        cases.append((f"quantised{S}", q))
    z = rng.random(3000, dtype=np.float32)
    z[:1000] = 0.0
    cases.append(("zeros_prefix", z))
    cases.append(("all_equal", np.full(777, 0.5, np.float32)))
    q = np.round(rng.random(5000) * 16).astype(np.float32)      # heavy ties
    cases.append(("quantised", q))
    last_low = rng.random(2000, dtype=np.float32)
    last_low[-1] = 0.0
    cases.append(("last_low", last_low))
    last_tie = np.round(rng.random(2000) * 4).astype(np.float32)
    last_tie[-1] = 2.0
    cases.append(("last_tie", last_tie))
    return cases


@pytest.mark.parametrize("name,dev", _topk_cases(), ids=lambda x: x if isinstance(x, str) else "")
@pytest.mark.parametrize("force", [False, True])
def test_topk_select_bit_exact(ops, name, dev, force):
    S = len(dev)
    for k in sorted({1, max(1, S // 10), hp.topk_count(S, 0.15), S}):
        st = status_word()
        got = ops.topk_select(torch.from_numpy(dev).to(DEV), k, force_last=force, status=st).cpu().numpy()
        assert_status_clean(st)
        np.testing.assert_array_equal(got, hp.topk_select(dev, k, force_last=force), err_msg=f"k={k}")


def test_select_top_k_api_vs_reference_golden():
    from cacheblend import select_top_k
    k = golden("kernels_bf16.npz")
    for r in (0.001, 0.1, 0.15, 0.5, 1.0):
        got = select_top_k(torch.from_numpy(k["dev_out"]).to(DEV), r)
        assert got.dtype == torch.int64 and got.device.type == "cuda"
        np.testing.assert_array_equal(got.cpu().numpy(), k[f"topk_{r}"])
    for n in (1, 7, 544, 6208):
        got = select_top_k(torch.from_numpy(k[f"topk_rand_{n}"]).to(DEV), 0.15).cpu().numpy()
        np.testing.assert_array_equal(got, k[f"topk_rand_{n}_idx"])
    from cacheblend import ops as o
    got = o.topk_select(torch.from_numpy(k["force_dev"]).to(DEV), hp.topk_count(200, 0.15),
                        force_last=True).cpu().numpy()
    np.testing.assert_array_equal(got, k["force_idx"])


def test_hkvd_select_fused(ops):
    g = torch.Generator().manual_seed(21)
    lengths = [1024] * 6 + [64]
    entries = _make_store(lengths, 2, 1024, "bf16", g)
    S = sum(lengths)
    old = torch.cat([e["K"][1][0] for e in entries]).cpu()
    new = (old.float() + torch.randn((S, 1024), generator=g) * 0.05).to(torch.bfloat16)
    table = ops.ChunkTable(entries, [0, 1], torch.device(DEV))
    k = hp.topk_count(S, 0.15)
    st = status_word()
    idx, dev = ops.hkvd_select(new.to(DEV), table, 1, k, force_last=True, status=st)
    assert_status_clean(st)
    exp_dev = hp.kv_deviation(bf16_to_f32(to_bits(new)), bf16_to_f32(to_bits(old)))
    np.testing.assert_array_equal(dev.cpu().numpy(), exp_dev)
    np.testing.assert_array_equal(idx.cpu().numpy(), hp.topk_select(exp_dev, k, force_last=True))


# ---------------------------------------------------------------------------
# (e) partial attention
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("case", ac.CASES, ids=[c[0] for c in ac.CASES])
def test_partial_attention(ops, case):
    """Element by element within tol * (|exp| + A) of the fp64 oracle (A: the
    softmax weights applied to |V|; tol 2^-7 bf16, 2^-9 fp16), and max |err|
    within 2e-2 of max |exp|.  Peaked cases (q scaled) make outputs O(1) and
    single keys decisive; big-V cases put |V| up to ~5e5 (bf16) and ~5.5e4 (fp16)
    through split tiles.  tests/test_attn_bound.py shows that an off-by-one
    causal bound, a dropped split chunk or a wrong merge weight violate this
    bound on the peaked cases."""
    name, S, n_sel, Hq, Hkv, D, dtype, _, _ = case
    q, k, v, pos = ac.make_inputs(case)
    st = status_word()
    out = ops.partial_attn(q.to(DEV), k.to(DEV), v.to(DEV), pos.to(DEV), Hq, Hkv, D, D ** -0.5,
                           status=st)
    assert_status_clean(st)
    got = DEC[dtype](to_bits(out))
    exp, absm = ac.oracle(case, q, k, v, pos)
    ac.check(got, exp, absm, dtype)


def test_partial_attention_vs_reference_golden(ops):
    k = golden("kernels_bf16.npz")
    q = from_bits(k["attn_q"]).transpose(0, 1).reshape(-1, 4 * 64).contiguous()
    kk = from_bits(k["attn_k"]).transpose(0, 1).reshape(-1, 2 * 64).contiguous()
    v = from_bits(k["attn_v"]).transpose(0, 1).reshape(-1, 2 * 64).contiguous()
    pos = torch.from_numpy(k["attn_pos"])
    out = ops.partial_attn(q.to(DEV), kk.to(DEV), v.to(DEV), pos.to(DEV), 4, 2, 64, 64 ** -0.5)
    ref = bf16_to_f32(k["attn_out"]).transpose(1, 0, 2).reshape(len(pos), -1)
    assert np.abs(bf16_to_f32(to_bits(out)) - ref).max() < 2e-2


def test_partial_attention_repeatable(ops):
    """Same inputs, same bits (no atomics / data races in the kernel)."""
    g = torch.Generator().manual_seed(77)
    S, n, Hq, Hkv, D = 3000, 400, 32, 8, 128
    pos = torch.sort(torch.randperm(S, generator=g)[:n]).values.to(DEV)
    q, k, v = (rand16(s, "bf16", g).to(DEV) for s in ((n, Hq * D), (S, Hkv * D), (S, Hkv * D)))
    a = ops.partial_attn(q, k, v, pos, Hq, Hkv, D, D ** -0.5)
    b = ops.partial_attn(q, k, v, pos, Hq, Hkv, D, D ** -0.5)
    assert torch.equal(a, b)


def test_partial_attention_plan_reuse(ops):
    """One plan (built from pos) serves every layer with the same selection: a
    second layer's inputs with reuse_plan give the same bits as a fresh plan."""
    g = torch.Generator().manual_seed(5)
    S, n, Hq, Hkv, D = 6208, 931, 32, 8, 128
    pos = torch.cat([torch.sort(torch.randperm(S - 1, generator=g)[:n - 1]).values,
                     torch.tensor([S - 1])]).to(DEV)
    layers = [tuple(rand16(sh, "bf16", g).to(DEV) for sh in ((n, Hq * D), (S, Hkv * D), (S, Hkv * D)))
              for _ in range(2)]
    ws = ops.attn_workspace(n, S, Hq, Hkv, D, DEV)
    st = status_word()
    a0 = ops.partial_attn(*layers[0], pos, Hq, Hkv, D, D ** -0.5, workspace=ws, reuse_plan=False, status=st)
    a1 = ops.partial_attn(*layers[1], pos, Hq, Hkv, D, D ** -0.5, workspace=ws, reuse_plan=True, status=st)
    b1 = ops.partial_attn(*layers[1], pos, Hq, Hkv, D, D ** -0.5)
    assert_status_clean(st)
    assert torch.equal(a1, b1)
    assert not torch.equal(a0, a1)
