"""Decoder-layer row kernels (cbk_add_rmsnorm, cbk_silu_mul) against the HF
modules they replace, run on the same GPU tensors.

The residual add and SiLU * up are the same fp32 operations with the same
16-bit roundings as torch: bit-exact.  RMSNorm sums the squares in a fixed
order that differs from torch's reduction, so the mean may move by an fp32 ulp;
the normalised value then rounds differently in rare elements (at most one
16-bit ulp), and the product with a weight up to ~1.5 keeps that within two
ulps of the output, in fewer than 1e-3 of the elements.  The fp32 restatement
of the norm bounds both the same way."""
import numpy as np
import pytest
import torch

from helpers import to_bits, ulp_diff_bf16

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _hf_norm(hidden, eps, dtype):
    from transformers.models.mistral.modeling_mistral import MistralRMSNorm
    m = MistralRMSNorm(hidden, eps=eps).to(DEV)
    with torch.no_grad():
        m.weight.copy_(1 + 0.1 * torch.randn(hidden, generator=torch.Generator().manual_seed(7)))
    return m.to(dtype)


def _ulps(a, b, dtype):
    if dtype == torch.bfloat16:
        return ulp_diff_bf16(to_bits(a), to_bits(b))
    ia = a.view(torch.int16).cpu().numpy().astype(np.int32)
    ib = b.view(torch.int16).cpu().numpy().astype(np.int32)
    return np.abs(ia - ib)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rows,hidden", [(1, 4096), (300, 4096), (931, 4096), (64, 8192), (17, 256)])
def test_add_rmsnorm_matches_hf_module(dtype, rows, hidden):
    from cacheblend import ops
    g = torch.Generator(device=DEV).manual_seed(rows + hidden)
    x = (torch.randn((1, rows, hidden), generator=g, device=DEV) * 3).to(dtype)
    d = torch.randn((1, rows, hidden), generator=g, device=DEV).to(dtype)
    norm = _hf_norm(hidden, 1e-5, dtype)
    with torch.inference_mode():
        ref_sum = x + d
        ref = norm(ref_sum)
        s = torch.empty_like(x)
        out = ops.add_rmsnorm(x, norm.weight, norm.variance_epsilon, delta=d, sum_out=s)
        plain = ops.add_rmsnorm(x, norm.weight, norm.variance_epsilon)
        ref_plain = norm(x)
    torch.cuda.synchronize()
    assert torch.equal(s, ref_sum)                        # residual add: bit-exact
    for got, exp in ((out, ref), (plain, ref_plain)):
        u = _ulps(got, exp, dtype)
        assert u.max() <= 2 and (u != 0).mean() < 1e-3, (u.max(), (u != 0).mean())


def test_add_rmsnorm_in_place_and_gather():
    from cacheblend import ops
    dtype, S, k, hidden = torch.bfloat16, 6208, 931, 4096
    g = torch.Generator(device=DEV).manual_seed(1)
    h = torch.randn((1, S, hidden), generator=g, device=DEV).to(dtype)
    idx = torch.sort(torch.randperm(S, generator=g, device=DEV)[:k])[0]
    o = torch.randn((1, k, hidden), generator=g, device=DEV).to(dtype)
    norm = _hf_norm(hidden, 1e-5, dtype)
    with torch.inference_mode():
        ref_sum = h.index_select(1, idx) + o
        ref = norm(ref_sum)
        hs = torch.empty_like(o)
        out = ops.add_rmsnorm(h, norm.weight, norm.variance_epsilon, delta=o, rows=idx, sum_out=hs)
        # in place: the residual stream is overwritten with its sum
        h2 = h.clone()
        d2 = torch.randn((1, S, hidden), generator=g, device=DEV).to(dtype)
        ref2_sum = h2 + d2
        ref2 = norm(ref2_sum)
        out2 = ops.add_rmsnorm(h2, norm.weight, norm.variance_epsilon, delta=d2, sum_out=h2)
    torch.cuda.synchronize()
    assert torch.equal(hs, ref_sum) and torch.equal(h2, ref2_sum)
    for got, exp in ((out, ref), (out2, ref2)):
        u = _ulps(got, exp, dtype)
        assert u.max() <= 2 and (u != 0).mean() < 1e-3
    with pytest.raises(ValueError):
        ops.add_rmsnorm(h, norm.weight, 1e-5, delta=o, rows=idx, sum_out=h[:, :k])


def test_add_rmsnorm_against_fp32_restatement():
    """The same formula in fp32 numpy with torch's 16-bit rounding points."""
    from cacheblend import ops
    from oracle.bf16 import bf16_to_f32, f32_to_bf16
    g = torch.Generator(device=DEV).manual_seed(5)
    x = torch.randn((64, 4096), generator=g, device=DEV).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(4096, generator=g, device=DEV)).to(torch.bfloat16)
    out = ops.add_rmsnorm(x, w, 1e-5)
    xf = bf16_to_f32(to_bits(x)).astype(np.float64)
    r = 1.0 / np.sqrt((xf * xf).mean(-1, keepdims=True) + 1e-5)
    y = bf16_to_f32(f32_to_bf16((xf * r).astype(np.float32)))
    exp = f32_to_bf16((bf16_to_f32(to_bits(w)) * y).astype(np.float32))
    u = ulp_diff_bf16(to_bits(out), exp)
    assert u.max() <= 2 and (u != 0).mean() < 1e-3


def test_add_rmsnorm_bad_index_sets_status():
    from cacheblend import _native as N, ops
    x = torch.randn((8, 256), device=DEV).to(torch.bfloat16)
    w = torch.ones(256, device=DEV, dtype=torch.bfloat16)
    rows = torch.tensor([0, 3, 8, 1], device=DEV)          # 8 is out of range
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = torch.zeros((4, 256), device=DEV, dtype=torch.bfloat16)
    ops.add_rmsnorm(x, w, 1e-5, rows=rows, out=out, status=st)
    torch.cuda.synchronize()
    assert int(st.item()) & N.CBK_STATUS_BAD_INDEX
    assert torch.all(out[2] == 0)                           # the bad row is left untouched
    ref = ops.add_rmsnorm(x[[0, 3, 1]], w, 1e-5)
    assert torch.equal(out[[0, 1, 3]], ref)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rows,cols", [(1, 14336), (931, 14336), (7, 8)])
def test_silu_mul_bit_exact_vs_torch(dtype, rows, cols):
    from cacheblend import ops
    g = torch.Generator(device=DEV).manual_seed(rows)
    gate = (torch.randn((1, rows, cols), generator=g, device=DEV) * 4).to(dtype)
    up = torch.randn((1, rows, cols), generator=g, device=DEV).to(dtype)
    gate.view(-1)[:4] = torch.tensor([0.0, -0.0, 30.0, -30.0], dtype=dtype)
    with torch.inference_mode():
        ref = torch.nn.functional.silu(gate) * up
        out = ops.silu_mul(gate, up)
    assert torch.equal(out, ref)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_silu_every_16bit_input(dtype):
    """The activation depends on the gate's 16 bits alone: all 65536 of them
    against torch's own SiLU kernel (up = 1, so the output is the rounded
    activation), NaN inputs giving NaN."""
    from cacheblend import ops
    bits = torch.arange(-32768, 32768, dtype=torch.int32, device=DEV).to(torch.int16)
    gate = bits.view(dtype).reshape(1, 256, 256)
    up = torch.ones_like(gate)
    with torch.inference_mode():
        ref = torch.nn.functional.silu(gate)
        out = ops.silu_mul(gate, up)
    nan = torch.isnan(ref)
    assert torch.equal(torch.isnan(out), nan)
    assert torch.equal(out.view(torch.int16)[~nan], ref.view(torch.int16)[~nan])


def test_silu_mul_strided_halves():
    """gate and up as the two halves of one wider row (a merged projection)."""
    from cacheblend import ops
    g = torch.Generator(device=DEV).manual_seed(9)
    gu = torch.randn((50, 2 * 1024), generator=g, device=DEV).to(torch.bfloat16)
    gate, up = gu[:, :1024], gu[:, 1024:]
    with torch.inference_mode():
        assert torch.equal(ops.silu_mul(gate, up), torch.nn.functional.silu(gate) * up)


@pytest.mark.parametrize("S,k,V,dtype", [(544, 81, 1000, torch.bfloat16), (6208, 931, 32000, torch.bfloat16),
                                         (100, 100, 512, torch.float32), (50, 1, 64, torch.float16),
                                         (10, 0, 64, torch.bfloat16)])
def test_scatter_rows_dense_logits(S, k, V, dtype):
    """ops.scatter_rows == torch zeros + index_copy_ (the reference's dense logits), bit for bit."""
    from cacheblend import ops
    g = torch.Generator(device=DEV).manual_seed(S + k)
    idx = torch.sort(torch.randperm(S, generator=g, device=DEV)[:k])[0]
    src = torch.randn((k, V), generator=g, device=DEV).to(dtype)
    ref = torch.zeros((S, V), dtype=dtype, device=DEV)
    ref.index_copy_(0, idx, src)
    out = torch.full((S, V), 7.0, dtype=dtype, device=DEV)       # every byte must be rewritten
    ops.scatter_rows(src, idx, S, out=out)
    assert torch.equal(out, ref)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("n,k", [(4096, 4096), (300, 14336), (33, 1000), (5, 8)])
def test_gemv_one_row(dtype, n, k):
    """ops.gemv against an fp64 product of the same 16-bit inputs: within half
    a 16-bit ulp of the result plus the fp32 accumulation error."""
    from cacheblend import ops
    g = torch.Generator(device=DEV).manual_seed(n + k)
    w = (torch.randn((n, k), generator=g, device=DEV) * 0.05).to(dtype)
    x = torch.randn((1, 1, k), generator=g, device=DEV).to(dtype)
    y = ops.gemv(w, x)
    assert y.shape == (1, 1, n) and y.dtype == dtype
    ref = w.double() @ x.view(-1).double()
    mag = w.double().abs() @ x.view(-1).double().abs()
    ulp = 2.0 ** (-8 if dtype == torch.bfloat16 else -11)
    # (fp16 results below 2^-14 are subnormal: their rounding step is 2^-24 absolute)
    bound = ref.abs() * ulp + mag * (k * 2.0 ** -23) + (2.0 ** -24 if dtype == torch.float16 else 1e-30)
    assert torch.all((y.view(-1).double() - ref).abs() <= bound)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_gemv_with_silu_mul_input(dtype):
    """gate/up given: the same bits as silu_mul followed by the plain GEMV."""
    from cacheblend import ops
    g = torch.Generator(device=DEV).manual_seed(7)
    inter, n = 2048, 512
    gu = (torch.randn((1, 1, 2 * inter), generator=g, device=DEV) * 3).to(dtype)
    w = (torch.randn((n, inter), generator=g, device=DEV) * 0.05).to(dtype)
    fused = ops.gemv(w, gate=gu[..., :inter], up=gu[..., inter:])
    plain = ops.gemv(w, ops.silu_mul(gu[..., :inter], gu[..., inter:]))
    assert torch.equal(fused, plain)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("hq,hkv,d,cap,p,qs", [(32, 8, 128, 6240, 6208, 1.0), (32, 8, 128, 6240, 0, 1.0),
                                              (32, 8, 128, 6240, 255, 1.0), (32, 8, 128, 6240, 6239, 1.0),
                                              (8, 8, 64, 700, 333, 1.0), (16, 2, 128, 300, 299, 1.0),
                                              (16, 4, 64, 40000, 39001, 1.0), (8, 4, 128, 5000, 4097, 1.0),
                                              (32, 4, 128, 131328, 131071, 1.0),
                                              (32, 8, 128, 6240, 6208, 8.0), (32, 4, 128, 131328, 131071, 6.0)])
def test_decode_attn_one_token(dtype, hq, hkv, d, cap, p, qs):
    """decode_attn against an fp64 softmax attention of the same 16-bit inputs
    over rows 0..p (rows past p hold garbage that must stay invisible).  The
    kernel works in fp32 and rounds once: element by element
    |err| <= tol * (|exp| + A), A the softmax weights applied to |V|, tol 2^-8
    (bf16) / 2^-10 (fp16), twice the output rounding.  qs scales q: 8 makes the
    softmax peaked (outputs O(1), single keys decisive)."""
    from cacheblend import ops
    g = torch.Generator(device=DEV).manual_seed(cap + p)
    q = (torch.randn((hq * d,), generator=g, device=DEV) * qs).to(dtype)
    kc = torch.randn((cap, hkv * d), generator=g, device=DEV).to(dtype)
    vc = torch.randn((cap, hkv * d), generator=g, device=DEV).to(dtype)
    pos = torch.tensor([p], dtype=torch.int64, device=DEV)
    ws = ops.decode_workspace(cap, hq, hkv, d, DEV)
    scale = d ** -0.5
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    for _ in range(2):                       # the workspace is reusable
        out = ops.decode_attn(q, kc, vc, pos, hq, hkv, d, scale, ws, status=st)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    G = hq // hkv
    qh = q.double().view(hkv, G, d)                       # q head hq = kv head hq // G
    k = kc[: p + 1].double().view(p + 1, hkv, d)
    v = vc[: p + 1].double().view(p + 1, hkv, d)
    w = torch.softmax(torch.einsum("kgd,jkd->kgj", qh, k) * scale, dim=-1)
    ref = torch.einsum("kgj,jkd->kgd", w, v).reshape(1, -1)
    absm = torch.einsum("kgj,jkd->kgd", w, v.abs()).reshape(1, -1)
    tol = 2.0 ** (-8 if dtype == torch.bfloat16 else -10)
    ratio = (out.double() - ref).abs() / (ref.abs() + absm)
    assert torch.isfinite(out).all()
    assert ratio.max().item() <= tol, (ratio.max().item(), (out.double() - ref).abs().max().item())


def test_decode_attn_bad_position_reported():
    from cacheblend import _native as N, ops
    q = torch.randn((32 * 128,), device=DEV).to(torch.bfloat16)
    kc = torch.randn((100, 8 * 128), device=DEV).to(torch.bfloat16)
    ws = ops.decode_workspace(100, 32, 8, 128, DEV)
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = torch.zeros((1, 32 * 128), device=DEV, dtype=torch.bfloat16)
    ops.decode_attn(q, kc, kc, torch.tensor([100], device=DEV), 32, 8, 128, 0.1, ws, out=out, status=st)
    torch.cuda.synchronize()
    assert int(st.item()) & N.CBK_STATUS_BAD_INDEX and torch.all(out == 0)
