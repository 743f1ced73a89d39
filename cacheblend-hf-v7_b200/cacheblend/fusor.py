"""Fusion strategies (API of cacheblend-hf-v7 ``fusor.py``).

``fuse_selective`` is CacheBlend's selective KV recompute, with its five
data-parallel stages on the sm_100a kernels:

  (a)+(b) ``assemble_kernel``   chunk K/V of every cached layer gathered into one
          token-major fused cache [L][S][Hkv*D], K rotated to its fused
          position in the same pass (one launch for all layers, on a side
          stream that overlaps the dense layers before the check layer);
  (c)     ``deviation_kernel`` + ``topk_kernel``  HKVD at the check layer,
          force-include of the last position on the device (no host sync);
  (b)+(d) ``rope_scatter_kernel``  RoPE of the fresh Q/K rows and their
          scatter into the fused cache, per layer;
  (e)     ``partial_attn_kernel``  selected queries against the full fused KV
          on tcgen05 tensor cores (causal by position, GQA without expansion).

Projections stay in the HF modules (cuBLAS through torch).  RMSNorm with the
residual add folded in, and SiLU(gate) * up, run as one-pass libcbk kernels
with the HF modules' 16-bit roundings (``add_rmsnorm``, ``silu_mul``); the
check layer's residual gather rides in the same norm launch.
The returned cache holds views of the fused buffers (no staging copy).
``fuse_full_recompute`` / ``fuse_full_reuse`` / ``fuse_prefix_cache`` keep the
reference's behaviour (they are the ratio==0 / ratio>=1 / single-chunk
shortcuts of ``fuse_selective``) and run through the HF forward.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from cacheblend import ops
from cacheblend.chunker import Chunk, chunk_offsets, fused_input_ids
from cacheblend.kv_store import KVStore
from cacheblend.model import LayerwiseOutput, attach_cache_layers, new_dynamic_cache
from cacheblend.rope import rope_table_for


def fuse_full_recompute(layerwise_model, chunks: list[Chunk], return_layerwise_output: bool = False):
    """Plain prefill over the fused ids (reference fusor.py:25-38)."""
    ids = fused_input_ids(chunks, device=layerwise_model.device)
    with torch.inference_mode():
        out = layerwise_model.forward_layerwise(input_ids=ids, use_cache=True)
    return out if return_layerwise_output else out.logits


def _store_entries(kv_store: KVStore, chunks, who: str):
    entries = []
    for c in chunks:
        if not kv_store.has(c.chunk_id):
            raise KeyError(f"{who}: chunk {c.chunk_id!r} not in KVStore")
        entries.append(kv_store.get(c.chunk_id))
    return entries


def _run_with_kv_hooks(layerwise_model, chunks, k_for_layer, v_for_layer, return_layerwise_output):
    handles = []
    for li, layer in enumerate(layerwise_model._inner.layers):
        handles.append(layer.self_attn.k_proj.register_forward_hook(
            lambda _m, _i, out, _li=li: k_for_layer(_li, out)))
        handles.append(layer.self_attn.v_proj.register_forward_hook(
            lambda _m, _i, out, _li=li: v_for_layer(_li, out)))
    try:
        return fuse_full_recompute(layerwise_model, chunks, return_layerwise_output)
    finally:
        for h in handles:
            h.remove()


def fuse_full_reuse(layerwise_model, chunks: list[Chunk], kv_store: KVStore,
                    return_layerwise_output: bool = False):
    """Every chunk token reuses its stored pre-RoPE K and V; HF RoPE then places
    them at fused positions (reference fusor.py:41-117)."""
    if len(chunks) <= 1:
        return fuse_full_recompute(layerwise_model, chunks, return_layerwise_output)
    entries = _store_entries(kv_store, chunks, "fuse_full_reuse")
    K = [torch.cat([e["K"][l] for e in entries], dim=1) for l in range(layerwise_model.num_layers)]
    V = [torch.cat([e["V"][l] for e in entries], dim=1) for l in range(layerwise_model.num_layers)]
    return _run_with_kv_hooks(layerwise_model, chunks, lambda l, _o: K[l], lambda l, _o: V[l],
                              return_layerwise_output)


def fuse_prefix_cache(layerwise_model, chunks: list[Chunk], kv_store: KVStore,
                      return_layerwise_output: bool = False):
    """Only the first chunk's K/V come from the store (reference fusor.py:120-185)."""
    if len(chunks) <= 1:
        return fuse_full_recompute(layerwise_model, chunks, return_layerwise_output)
    first = chunks[0]
    if not kv_store.has(first.chunk_id):
        raise KeyError(f"fuse_prefix_cache: first chunk {first.chunk_id!r} not in KVStore")
    entry = kv_store.get(first.chunk_id)
    n0 = first.length

    def patch(src):
        def f(l, out):
            res = out.clone()
            res[:, :n0, :] = src[l]
            return res
        return f
    return _run_with_kv_hooks(layerwise_model, chunks, patch(entry["K"]), patch(entry["V"]),
                              return_layerwise_output)


# ---------------------------------------------------------------------------
# selective recompute
# ---------------------------------------------------------------------------
def _side_stream(layerwise_model, device):
    s = getattr(layerwise_model, "_cbk_side_stream", None)
    if s is None or s.device != device:
        s = torch.cuda.Stream(device=device)
        try:
            layerwise_model._cbk_side_stream = s
        except AttributeError:
            pass
    return s


class _Geometry:
    def __init__(self, layerwise_model):
        attn0 = layerwise_model._inner.layers[0].self_attn
        cfg = attn0.config
        self.n_kv = cfg.num_key_value_heads
        self.n_q = cfg.num_attention_heads
        self.head_dim = attn0.head_dim
        self.kv_dim = self.n_kv * self.head_dim
        self.q_dim = self.n_q * self.head_dim
        self.scaling = float(attn0.scaling)


_RMSNORMS = ("MistralRMSNorm", "LlamaRMSNorm")
_MLPS = ("MistralMLP", "LlamaMLP")
_SILUS = ("SiLUActivation", "SiLU")


def _norm(mod, x, delta=None, rows=None, sum_out=None, status=None):
    """mod(x[rows] + delta), also writing the sum to sum_out: the decoder
    layer's residual add plus its RMSNorm (MistralDecoderLayer.forward)."""
    if type(mod).__name__ in _RMSNORMS and mod.weight.dtype == x.dtype:
        return ops.add_rmsnorm(x, mod.weight, mod.variance_epsilon, delta=delta, rows=rows,
                               sum_out=sum_out, status=status)
    s = x if rows is None else x.index_select(x.dim() - 2, rows)
    if delta is not None:
        s = s + delta
    if sum_out is not None:
        sum_out.copy_(s)
    return mod(s)


# Row counts up to which the stacked q/k/v and gate/up GEMMs run (measured with
# cuBLAS bf16 at Mistral-7B shapes: 931 rows 32.5 us for q/k/v stacked vs 41.8
# separate, gate/up 155 vs 158; one decode row 11.5 vs 48.4; 6208 rows the
# separate GEMMs are faster, 210 vs 227 and 955 vs 1046).
FUSED_PROJ_MAX_ROWS = 4096


def _fused_w(lw, li, rows):
    """The stacked (W_qkv, W_gate_up) of layer li for a GEMM over `rows` rows,
    (None, None) above FUSED_PROJ_MAX_ROWS."""
    if lw is None or rows > FUSED_PROJ_MAX_ROWS:
        return None, None
    return lw.fused_projections(li)


def _mlp(layer, hn, w_gu=None):
    mlp = layer.mlp
    if type(mlp).__name__ in _MLPS and type(mlp.act_fn).__name__ in _SILUS:
        if w_gu is not None:          # one GEMM, gate and up as column views of its output
            gu = F.linear(hn, w_gu)
            inter = mlp.gate_proj.weight.shape[0]
            return mlp.down_proj(ops.silu_mul(gu[..., :inter], gu[..., inter:]))
        return mlp.down_proj(ops.silu_mul(mlp.gate_proj(hn), mlp.up_proj(hn)))
    return mlp(hn)


def _qkv(attn, hn, w_qkv=None):
    if w_qkv is None:
        return attn.q_proj(hn), attn.k_proj(hn), attn.v_proj(hn)
    qkv = F.linear(hn, w_qkv)         # one GEMM, q / k / v as column views of its output
    nq, nk = attn.q_proj.weight.shape[0], attn.k_proj.weight.shape[0]
    return qkv[..., :nq], qkv[..., nq:nq + nk], qkv[..., nq + nk:]


def _attention_block(layer, geo, hn, pos, S, rope, kc, vc, gather, status, rope_mode, ws, reuse,
                     tag="", w_qkv=None, rope_by_row=False):
    """q/k/v projections -> (b)+(d) RoPE + scatter into the fused cache ->
    (e) partial attention -> o_proj.  Returns the attention output rows and the
    pre-RoPE K (which the k_proj hook records when k_proj runs on its own).
    ``rope_by_row``: ``rope`` holds the cos/sin of pos[j] in row j."""
    attn = layer.self_attn
    q, k_pre, v = _qkv(attn, hn, w_qkv)
    q_rot = ops.rope_scatter(q[0], k_pre[0], v[0], pos, gather, S, geo.n_q, geo.n_kv, geo.head_dim,
                             rope, kc, vc, mode=rope_mode, status=status, table_by_row=rope_by_row)
    a = ops.partial_attn(q_rot, kc, vc, pos, geo.n_q, geo.n_kv, geo.head_dim, geo.scaling,
                         status=status, workspace=ws, reuse_plan=reuse, timer_tag=tag)
    return attn.o_proj(a.unsqueeze(0)), k_pre


_LOGITS_ROWS = ("all", "last")


def fuse_selective(layerwise_model, chunks: list[Chunk], kv_store: KVStore,
                   recompute_ratio: float = 0.15, check_layer: int = 1,
                   return_layerwise_output: bool = False, return_hkvd_indices: bool = False,
                   rope_mode: str = "ref", status: torch.Tensor | None = None,
                   input_ids: torch.Tensor | None = None, logits_rows: str = "all",
                   cuda_graph: bool | None = None):
    """CacheBlend selective recompute (reference fusor.py:193-497).

    Layers < check_layer: full forward.  Check layer: HKVD picks the
    max(1, int(S * ratio)) tokens whose fresh pre-RoPE K deviates most from the
    cached K (the last position is always included); from there on only those
    rows are recomputed, against the full fused cache (cached, RoPE-shifted K/V
    elsewhere).  Returns logits (1, S, vocab) with rows outside the selection
    zero, or a LayerwiseOutput with the full-length cache; optionally the
    selected indices.

    ``rope_mode`` "ref" reproduces HF's 16-bit RoPE rounding, "fp32" rotates in
    fp32 with one rounding.  ``status`` (int32 CUDA tensor) collects device-side
    error bits.  ``input_ids`` (1-D or (1, S) int64, host -- preferably pinned --
    or device) replaces the ids gathered from ``chunks``.

    ``logits_rows``: "all" (default) returns the reference's dense (1, S, vocab)
    logits; "last" runs the final norm and lm_head on the last position only and
    returns its logits as (1, 1, vocab) -- the only row a prefill's caller reads
    (fusor.py:486-491 fills the other selected rows, runners decode from
    [:, -1]); at 32K tokens and a 128K vocab the dense tensor is 8.4 GB.

    ``cuda_graph``: None (default) or True replays a CUDA graph of the selective
    path captured once per request geometry (chunk lengths, ratio, check layer,
    RoPE mode, logits rows) and kept on the model (the two most recent
    geometries); the first call of a geometry runs the path eagerly twice and
    captures it.  Results are bit-identical to the eager path (False), and
    every call returns new tensors.  After a replayed call the pre-RoPE K that
    ``get_pre_rope_k`` returns lives in the graph's memory and is overwritten
    by the next call of the same geometry."""
    if recompute_ratio == 0:
        return fuse_full_reuse(layerwise_model, chunks, kv_store, return_layerwise_output)
    if recompute_ratio >= 1:
        return fuse_full_recompute(layerwise_model, chunks, return_layerwise_output)
    if len(chunks) <= 1:
        return fuse_full_recompute(layerwise_model, chunks, return_layerwise_output)
    if logits_rows not in _LOGITS_ROWS:
        raise ValueError(f"logits_rows must be one of {_LOGITS_ROWS}, got {logits_rows!r}")
    if not 0 <= int(check_layer) < layerwise_model.num_layers:
        raise IndexError(f"check_layer {check_layer} out of range for {layerwise_model.num_layers} layers")
    graph = None
    if cuda_graph is not False and _graphs_enabled(layerwise_model):
        graph = _cached_graph(layerwise_model, chunks, kv_store, recompute_ratio, check_layer, rope_mode,
                              logits_rows)
    if graph is not None:
        with torch.inference_mode():
            pre = graph.replay(chunks, kv_store, input_ids)
            layerwise_model._pre_rope_k = dict(graph.pre_rope_k)
            if status is not None:
                status.bitwise_or_(graph.status)
            logits = _fresh_logits(pre, logits_rows)
            idx = pre.idx.clone()
            result = logits
            if return_layerwise_output:
                own = _Prefill(logits, pre.fused_k.clone(), pre.fused_v.clone(), idx, pre.geo, pre.S, pre.rope)
                result = LayerwiseOutput(logits=logits, past_key_values=own.dynamic_cache())
    else:
        pre = _selective_prefill(layerwise_model, chunks, kv_store, recompute_ratio, check_layer, rope_mode,
                                 status, input_ids, extra_tokens=0, logits_rows=logits_rows)
        idx = pre.idx
        result = pre.logits
        if return_layerwise_output:
            result = LayerwiseOutput(logits=pre.logits, past_key_values=pre.dynamic_cache())
    if return_hkvd_indices:
        return result, idx
    return result


# CUDA graphs of the selective path, per model and request geometry
GRAPH_CACHE_SIZE = 2


def _graphs_enabled(lw) -> bool:
    import os
    if os.environ.get("CACHEBLEND_CUDA_GRAPH", "1") == "0":
        return False
    if getattr(lw, "device", torch.device("cpu")).type != "cuda":
        return False
    return not torch.cuda.is_current_stream_capturing()


def _cached_graph(lw, chunks, kv_store, ratio, ck, rope_mode, logits_rows):
    """The model's captured graph of this geometry (captured on first use), or
    None when the path could not be captured (then the eager path runs)."""
    from collections import OrderedDict
    from cacheblend.graph import BlendGraph
    cache = getattr(lw, "_cbk_graphs", None)
    if cache is None:
        cache = OrderedDict()
        try:
            lw._cbk_graphs = cache
        except AttributeError:
            return None
    key = (tuple(c.length for c in chunks), float(ratio), int(ck), rope_mode, logits_rows, str(lw.device))
    if key in cache:
        cache.move_to_end(key)
        return cache[key]
    try:
        g = BlendGraph(lw, chunks, kv_store, ratio, ck, rope_mode, logits_rows=logits_rows, dense_logits=False)
    except (KeyError, ValueError, IndexError, NotImplementedError):
        raise                              # the caller's error, as the eager path raises it
    except RuntimeError:
        g = None                           # not capturable here: eager from now on
    cache[key] = g
    while len(cache) > GRAPH_CACHE_SIZE:
        cache.popitem(last=False)
    return g


def release_graphs(layerwise_model) -> None:
    """Drop the CUDA graphs fuse_selective keeps on the model (and their memory)."""
    cache = getattr(layerwise_model, "_cbk_graphs", None)
    if cache is not None:
        cache.clear()


def _fresh_logits(pre, logits_rows):
    """New logits tensor from a prefill's selected-row logits."""
    ls = pre.logits_sparse
    if logits_rows == "last":
        return ls.clone()
    return _dense_logits(ls, pre.idx, pre.S)


def _dense_logits(logits_sparse, idx, S):
    """(1, S, vocab) with the selected rows' logits and zeros elsewhere, one write
    pass (rows whose byte length is not a multiple of 16 take torch's zeros +
    index_copy_)."""
    if (logits_sparse.shape[-1] * logits_sparse.element_size()) % 16 == 0:
        return ops.scatter_rows(logits_sparse[0], idx, S).unsqueeze(0)
    logits = torch.zeros((1, S, logits_sparse.shape[-1]), dtype=logits_sparse.dtype, device=logits_sparse.device)
    logits[0].index_copy_(0, idx, logits_sparse[0])
    return logits


class _Prefill:
    """Result of a selective prefill: logits, the fused cache (capacity S + extra
    rows per layer, the first S filled) and the selection."""

    def __init__(self, logits, fused_k, fused_v, idx, geo, S, rope, logits_sparse=None):
        self.logits, self.fused_k, self.fused_v, self.idx = logits, fused_k, fused_v, idx
        self.geo, self.S, self.rope = geo, S, rope
        self.logits_sparse = logits_sparse      # (1, k or 1, vocab): the rows lm_head ran on

    def dynamic_cache(self):
        g, S = self.geo, self.S
        kv = [(self.fused_k[l, :S].view(S, g.n_kv, g.head_dim).permute(1, 0, 2).unsqueeze(0),
               self.fused_v[l, :S].view(S, g.n_kv, g.head_dim).permute(1, 0, 2).unsqueeze(0))
              for l in range(self.fused_k.shape[0])]
        return attach_cache_layers(new_dynamic_cache(), kv)


def _selective_prefill(layerwise_model, chunks, kv_store, recompute_ratio, check_layer, rope_mode, status,
                       input_ids, extra_tokens: int = 0, table=None, logits_rows: str = "all",
                       dense_logits: bool = True) -> _Prefill:
    """Body of fuse_selective's selective path; the fused cache gets extra_tokens
    spare rows per layer (room for decode).  ``table``: a prebuilt chunk table
    of layers check_layer.. (a captured graph keeps one and refreshes it).
    ``logits_rows`` "last": lm_head on the last position only; with
    ``dense_logits`` False the (1, S, vocab) tensor is not formed (the caller
    forms it from ``logits_sparse``)."""
    lw = layerwise_model
    inner = lw._inner
    n_layers = lw.num_layers
    ck = int(check_layer)
    if not 0 <= ck < n_layers:
        raise IndexError(f"check_layer {ck} out of range for {n_layers} layers")
    device = lw.device
    if device.type != "cuda":
        raise RuntimeError("fuse_selective runs on the sm_100a kernels: the model must be on CUDA")
    dtype = lw.dtype
    ops.dtype_code(dtype)
    geo = _Geometry(lw)

    entries = _store_entries(kv_store, chunks, "fuse_selective")
    offsets = chunk_offsets(chunks)
    S = offsets[-1][1]
    k_sel = max(1, min(S, int(S * recompute_ratio)))
    cur = torch.cuda.current_stream(device)

    with torch.inference_mode():
        if table is None:
            table = ops.ChunkTable(entries, range(ck, n_layers), device)
        if table.S != S:
            raise ValueError(f"stored chunk lengths sum to {table.S}, chunks say {S}")
        rope = rope_table_for(lw, S + extra_tokens, device)
        fused_k = torch.empty((n_layers, S + extra_tokens, geo.kv_dim), dtype=dtype, device=device)
        fused_v = torch.empty_like(fused_k)
        fk, fv = fused_k[:, :S], fused_v[:, :S]     # the blended rows of every layer
        if extra_tokens:
            # spare rows hold zeros until decode writes them: attention over the whole
            # capacity multiplies P = 0 by them, and 0 * (uninitialised NaN) would not be 0
            fused_k[:, S:].zero_()
            fused_v[:, S:].zero_()

        # (a)+(b): all cached layers in one launch on a side stream.  It starts once the
        # last full layer's attention has been issued (at once when check_layer is 0),
        # so this HBM-bound copy overlaps that layer's MLP GEMMs and the check layer's
        # projections, and the attention kernel has the SMs to itself.
        side = _side_stream(lw, device)
        assembled = torch.cuda.Event()

        def launch_assemble():
            side.wait_stream(cur)
            with torch.cuda.stream(side):
                ops.assemble_kv(table, ck, n_layers, geo.n_kv, geo.head_dim, rope, fused_k, fused_v,
                                mode=rope_mode, status=status)
            assembled.record(side)
        # No record_stream: the current stream waits for `assembled` below, before
        # anything can free these buffers, so their memory returns to the caching
        # allocator in stream order.  (record_stream would hold it until the side
        # stream's event completes, and with the device running behind the host the
        # next blend could not reuse it and would allocate anew.)

        # the side stream writes fused_k / fused_v until `assembled`: whatever
        # happens below, the current stream is ordered after it before they can
        # be freed (waiting on an event that was never recorded is a no-op)
        if ck == 0:
            launch_assemble()
        try:
            if input_ids is None:
                ids = fused_input_ids(chunks, device=device)
            else:
                ids = input_ids.reshape(1, -1).to(device, non_blocking=True)
                if ids.shape[1] != S:
                    raise ValueError(f"input_ids has {ids.shape[1]} tokens, chunks have {S}")
            lw._pre_rope_k = {}
            pos_all = torch.arange(S, device=device, dtype=torch.int64)
            h = inner.embed_tokens(ids)     # residual stream; updated in place by the fused norms
            m = None                        # pending MLP output, added by the next norm

            ws_dense = ops.attn_workspace(S, S, geo.n_q, geo.n_kv, geo.head_dim, device) if ck else None
            for li in range(ck):                                  # dense layers (one shared plan)
                layer = inner.layers[li]
                hn = _norm(layer.input_layernorm, h, delta=m, sum_out=h if m is not None else None,
                           status=status)
                a, _ = _attention_block(layer, geo, hn, pos_all, S, rope,
                                        fk[li], fv[li], False, status, rope_mode, ws_dense, li > 0,
                                        tag="_dense")
                if li == ck - 1:
                    launch_assemble()
                m = _mlp(layer, _norm(layer.post_attention_layernorm, h, delta=a, sum_out=h, status=status))

            # check layer: full-row K, HKVD, then sparse from here on
            layer = inner.layers[ck]
            attn = layer.self_attn
            hn = _norm(layer.input_layernorm, h, delta=m, sum_out=h if m is not None else None, status=status)
            k_pre = attn.k_proj(hn)             # every row: HKVD compares each token's fresh K
            idx, deviations = ops.hkvd_select(k_pre[0], table, ck, k_sel, force_last=True, status=status)
            # Q and V only for the selected rows (the reference projects all S rows,
            # fusor.py:333-335, and keeps these)
            hn_sel = hn.index_select(1, idx)
            q = attn.q_proj(hn_sel)
            v = attn.v_proj(hn_sel)
            k_rows = k_pre.index_select(1, idx)
            # cos/sin of the selected positions, one row per selected token: every
            # later rope_scatter reads them without waiting for the positions
            rope_sel = rope.index_select(0, idx)
            cur.wait_event(assembled)
            q_rot = ops.rope_scatter(q[0], k_rows[0], v[0], idx, False, S, geo.n_q, geo.n_kv, geo.head_dim,
                                     rope_sel, fk[ck], fv[ck], mode=rope_mode, status=status, table_by_row=True)
            ws_sparse = ops.attn_workspace(k_sel, S, geo.n_q, geo.n_kv, geo.head_dim, device)
            a = ops.partial_attn(q_rot, fk[ck], fv[ck], idx, geo.n_q, geo.n_kv, geo.head_dim,
                                 geo.scaling, status=status, workspace=ws_sparse, reuse_plan=False)
            # selected residual rows gathered inside the norm launch
            o = attn.o_proj(a.unsqueeze(0))
            hs = torch.empty_like(o)
            m = _mlp(layer, _norm(layer.post_attention_layernorm, h, delta=o, rows=idx, sum_out=hs, status=status),
                     _fused_w(lw, ck, k_sel)[1])

            for li in range(ck + 1, n_layers):                    # sparse layers
                layer = inner.layers[li]
                w_qkv, w_gu = _fused_w(lw, li, k_sel)
                hn = _norm(layer.input_layernorm, hs, delta=m, sum_out=hs, status=status)
                a, k_pre = _attention_block(layer, geo, hn, idx, S, rope_sel, fk[li], fv[li], False, status,
                                            rope_mode, ws_sparse, True, w_qkv=w_qkv, rope_by_row=True)
                if w_qkv is not None:
                    lw._pre_rope_k[li] = k_pre
                m = _mlp(layer, _norm(layer.post_attention_layernorm, hs, delta=a, sum_out=hs, status=status),
                         w_gu)

            if logits_rows == "last":       # idx is ascending and holds S - 1: the last selected row
                hs_out = _norm(inner.norm, hs[:, -1:], delta=m[:, -1:], status=status)
            else:
                hs_out = _norm(inner.norm, hs, delta=m, status=status)
            logits_sparse = lw.model.lm_head(hs_out)            # (1, k or 1, vocab)
            if not dense_logits:
                logits = None
            elif logits_rows == "last":
                logits = logits_sparse
            else:
                logits = _dense_logits(logits_sparse, idx, S)
        finally:
            cur.wait_event(assembled)

    return _Prefill(logits, fused_k, fused_v, idx, geo, S, rope, logits_sparse)
