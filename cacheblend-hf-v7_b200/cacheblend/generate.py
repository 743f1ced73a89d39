"""Greedy decode over the blended cache (the decode loop of cacheblend-hf-v7's
runners, ``runners.py:106-152``) on the libcbk kernels.

The selective prefill keeps its fused cache with spare rows; each decode step
then runs the decoder for one token at position p: residual add + RMSNorm as
the fused row kernel, the projections as one-row GEMV kernels (q/k/v and
gate/up over the stacked weights, o, down and lm_head; SiLU * up by
``silu_mul``), RoPE of the token's Q and K with its K/V written
into cache row p (``rope_scatter`` with one index), and attention of the one
query row over rows [0, p] (``decode_attn``: split over the keys, HBM-bound).  Token 1 is the argmax of
the last prefill row, as in the reference; decoding stops after
``max_new_tokens`` tokens or at ``eos_token_id``.
"""
from __future__ import annotations

import torch

from cacheblend import ops
from cacheblend.chunker import Chunk
from cacheblend.fusor import _MLPS, _SILUS, _fused_w, _mlp, _norm, _qkv, _selective_prefill, fuse_selective
from cacheblend.kv_store import KVStore


class _DecodeState:
    """Static device buffers of a decode: the current token and position, the
    attention workspace, and the chosen tokens / logits rows by step."""

    def __init__(self, lw, pre, n_new: int, first_row: torch.Tensor, keep_rows: bool):
        device, geo = lw.device, pre.geo
        cap = pre.fused_k.shape[1]
        self.tokens = torch.zeros((n_new,), dtype=torch.int64, device=device)
        self.rows = torch.zeros((n_new, first_row.shape[-1]), dtype=first_row.dtype, device=device) if keep_rows else None
        first = first_row.argmax().view(1)
        self.tokens[0:1].copy_(first)
        if keep_rows:
            self.rows[0].copy_(first_row)
        self.token = first.view(1, 1).clone()
        self.pos = torch.full((1,), pre.S, dtype=torch.int64, device=device)
        self.base = pre.S - 1               # token t of the output was chosen at position base + t
        # one-token attention kernel where it applies (head_dim 64/128, 1, 2, 4 or 8 q heads
        # per KV head), else the selective-attention kernel with a one-row selection
        self.one_row = geo.head_dim in (64, 128) and geo.n_q // geo.n_kv in (1, 2, 4, 8)
        self.ws = (ops.decode_workspace(cap, geo.n_q, geo.n_kv, geo.head_dim, device) if self.one_row
                   else ops.attn_workspace(1, cap, geo.n_q, geo.n_kv, geo.head_dim, device))


def _gemv_ok(w: torch.Tensor, x: torch.Tensor) -> bool:
    return w.dtype == x.dtype and w.shape[1] % 8 == 0 and w.shape[1] <= 16384 and w.stride(1) == 1


def _lin1(mod, x):
    """A Linear at one decode row on the GEMV kernel (bias-free, the input's
    dtype), else the module itself."""
    if isinstance(mod, torch.nn.Linear) and mod.bias is None and _gemv_ok(mod.weight, x):
        return ops.gemv(mod.weight, x)
    return mod(x)


def _qkv1(attn, hn, w_qkv):
    if w_qkv is None or not _gemv_ok(w_qkv, hn):
        return _qkv(attn, hn, w_qkv)
    qkv = ops.gemv(w_qkv, hn)
    nq, nk = attn.q_proj.weight.shape[0], attn.k_proj.weight.shape[0]
    return qkv[..., :nq], qkv[..., nq:nq + nk], qkv[..., nq + nk:]


def _mlp1(layer, hn, w_gu):
    """MLP at one decode row: the stacked gate/up GEMV, SiLU * up, then the down GEMV."""
    mlp = layer.mlp
    down = getattr(mlp, "down_proj", None)
    if (w_gu is None or type(mlp).__name__ not in _MLPS or type(mlp.act_fn).__name__ not in _SILUS
            or not isinstance(down, torch.nn.Linear) or down.bias is not None or not _gemv_ok(w_gu, hn)
            or not _gemv_ok(down.weight, hn)):
        return _mlp(layer, hn, w_gu)
    gu = ops.gemv(w_gu, hn)
    inter = mlp.gate_proj.weight.shape[0]
    # one silu_mul launch, then the plain GEMV: 24.8 vs 26.3 us at 4096 x 14336 for
    # the GEMV forming SiLU * up itself (each of its CTAs stages the activation)
    return ops.gemv(down.weight, ops.silu_mul(gu[..., :inter], gu[..., inter:]))


def _decode_step(lw, pre, st: _DecodeState, status):
    """One token at position st.pos: its K/V into cache row pos, the next token
    into st.token / st.tokens, pos advanced -- all on the device, no host sync
    (so the step can be captured in a CUDA graph)."""
    inner, geo = lw._inner, pre.geo
    cap = pre.fused_k.shape[1]
    h = inner.embed_tokens(st.token)
    m = None
    for li, layer in enumerate(inner.layers):
        attn = layer.self_attn
        w_qkv, w_gu = _fused_w(lw, li, 1)      # one row: the stacked GEMMs
        hn = _norm(layer.input_layernorm, h, delta=m, sum_out=h if m is not None else None, status=status)
        q, k, v = _qkv1(attn, hn, w_qkv)
        q_rot = ops.rope_scatter(q[0], k[0], v[0], st.pos, False, cap, geo.n_q, geo.n_kv, geo.head_dim, pre.rope,
                                 pre.fused_k[li], pre.fused_v[li], status=status)
        # the whole capacity with the position as the causal bound: rows past pos are
        # invisible (and zero), so the call does not change from step to step
        if st.one_row:
            a = ops.decode_attn(q_rot, pre.fused_k[li], pre.fused_v[li], st.pos, geo.n_q, geo.n_kv, geo.head_dim,
                                geo.scaling, st.ws, status=status)
        else:
            # the plan depends on the position only: made by the first layer, reused by the rest
            a = ops.partial_attn(q_rot, pre.fused_k[li], pre.fused_v[li], st.pos, geo.n_q, geo.n_kv,
                                 geo.head_dim, geo.scaling, status=status, workspace=st.ws, reuse_plan=li > 0)
        o = _lin1(attn.o_proj, a.unsqueeze(0))
        m = _mlp1(layer, _norm(layer.post_attention_layernorm, h, delta=o, sum_out=h, status=status), w_gu)
    row = _lin1(lw.model.lm_head, _norm(inner.norm, h, delta=m, status=status))[0, -1]
    nxt = row.argmax().view(1)
    slot = st.pos - st.base
    st.tokens.index_copy_(0, slot, nxt)
    if st.rows is not None:
        st.rows.index_copy_(0, slot, row.view(1, -1))
    st.token.copy_(nxt.view(1, 1))
    st.pos.add_(1)


def generate_greedy(layerwise_model, chunks: list[Chunk], kv_store: KVStore, max_new_tokens: int,
                    recompute_ratio: float = 0.15, check_layer: int = 1, eos_token_id: int | None = None,
                    rope_mode: str = "ref", status: torch.Tensor | None = None, return_logits: bool = False,
                    use_graph: bool = True):
    """CacheBlend selective prefill, then greedy decode over the blended cache.

    Returns the generated token ids (token 1 from the prefill's last row), and
    with ``return_logits`` the logits row that chose each of them.  Decode
    steps run back to back on the device (one CUDA graph of a step, replayed,
    unless ``use_graph`` is False); the tokens are read once at the end and cut
    after the first ``eos_token_id``, so a run that meets EOS early decodes the
    remaining steps for nothing but returns what the reference returns.  The
    shortcut cases of fuse_selective (ratio 0, ratio >= 1, one chunk) run the
    reference path: HF prefill and HF decode with ``past_key_values``."""
    if max_new_tokens <= 0:
        return ([], []) if return_logits else []
    lw = layerwise_model
    selective = 0 < recompute_ratio < 1 and len(chunks) > 1
    tokens, rows = [], []
    with torch.inference_mode():
        if not selective:
            out = fuse_selective(lw, chunks, kv_store, recompute_ratio, check_layer, return_layerwise_output=True)
            row = out.logits[0, -1]
            cache = out.past_key_values
            for i in range(max_new_tokens):
                nxt = row.argmax()
                tokens.append(int(nxt.item()))
                rows.append(row)
                if (eos_token_id is not None and tokens[-1] == eos_token_id) or i + 1 == max_new_tokens:
                    break
                step = lw.model(input_ids=nxt.view(1, 1), past_key_values=cache, use_cache=True)
                cache, row = step.past_key_values, step.logits[0, -1]
        else:
            # only the last prefill row is read: lm_head on that row alone
            pre = _selective_prefill(lw, chunks, kv_store, recompute_ratio, check_layer, rope_mode, status,
                                     None, extra_tokens=max_new_tokens, logits_rows="last")
            st = _DecodeState(lw, pre, max_new_tokens, pre.logits[0, -1], return_logits)
            n_steps = max_new_tokens - 1
            if n_steps >= 1:
                _decode_step(lw, pre, st, status)          # eager: first use sets up every kernel
            if n_steps >= 2:
                if use_graph:
                    cur = torch.cuda.current_stream(lw.device)
                    side = torch.cuda.Stream(device=lw.device)
                    side.wait_stream(cur)
                    graph = torch.cuda.CUDAGraph()
                    with torch.cuda.stream(side):
                        with torch.cuda.graph(graph, stream=side):
                            _decode_step(lw, pre, st, status)
                    cur.wait_stream(side)
                    # capture recorded the step without running it
                    for _ in range(n_steps - 1):
                        graph.replay()
                    del graph
                else:
                    for _ in range(n_steps - 1):
                        _decode_step(lw, pre, st, status)
            tokens = st.tokens.tolist()
            if eos_token_id is not None and eos_token_id in tokens:
                tokens = tokens[:tokens.index(eos_token_id) + 1]
            rows = list(st.rows[:len(tokens)]) if return_logits else []
    return (tokens, rows) if return_logits else tokens
