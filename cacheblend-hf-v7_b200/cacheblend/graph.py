"""fuse_selective captured as one CUDA graph per request geometry.

A blended prefill has no host decisions once its inputs are on the device:
HKVD selects on the device, the attention plan is built on the device, every
shape follows from the chunk lengths, the recompute ratio and the check layer.
``BlendGraph`` runs the selective path twice eagerly (every kernel and cuBLAS
handle set up), captures a third run, and afterwards each call only refreshes
two static device buffers -- the chunk pointer table and the fused input ids --
and replays the graph: no per-kernel launches from Python.  The graph's
outputs (logits, selection, fused cache) live in its memory and are
overwritten by the next replay; ``fuse_selective`` keeps one graph per
geometry and copies what it returns out of them.

The chunk table is refreshed when the device addresses of the chunks' stored
tensors change (a pointer signature of the store entries, not object
identities, which Python reuses): an evicted and re-stored chunk, or other
chunks of the same lengths, point the table at their own tensors.
"""
from __future__ import annotations

import torch

from cacheblend import ops
from cacheblend.chunker import Chunk, chunk_offsets
from cacheblend.fusor import _LOGITS_ROWS, _selective_prefill, _store_entries
from cacheblend.kv_store import KVStore


class BlendGraph:
    def __init__(self, layerwise_model, chunks: list[Chunk], kv_store: KVStore, recompute_ratio: float = 0.15,
                 check_layer: int = 1, rope_mode: str = "ref", logits_rows: str = "all",
                 dense_logits: bool = True):
        if not (0 < recompute_ratio < 1) or len(chunks) <= 1:
            raise ValueError("BlendGraph captures the selective path: 0 < recompute_ratio < 1 and >= 2 chunks")
        if logits_rows not in _LOGITS_ROWS:
            raise ValueError(f"logits_rows must be one of {_LOGITS_ROWS}, got {logits_rows!r}")
        lw = self.lw = layerwise_model
        self.ratio, self.ck, self.mode = recompute_ratio, int(check_layer), rope_mode
        self.logits_rows, self.dense_logits = logits_rows, dense_logits
        self.lengths = [c.length for c in chunks]
        self.S = chunk_offsets(chunks)[-1][1]
        device = lw.device
        entries = _store_entries(kv_store, chunks, "BlendGraph")
        self.table = ops.ChunkTable(entries, range(self.ck, lw.num_layers), device)
        self._sig = ops.chunk_signature(entries, self.table.layers)
        self.ids = torch.tensor([[t for c in chunks for t in c.token_ids]], dtype=torch.int64, device=device)
        self.status = torch.zeros(1, dtype=torch.int32, device=device)
        cur = torch.cuda.current_stream(device)
        side = torch.cuda.Stream(device=device)
        side.wait_stream(cur)
        with torch.inference_mode(), torch.cuda.stream(side):
            for _ in range(2):                       # warm-up: kernels, handles, allocator pools
                self._run(chunks, kv_store)
            side.synchronize()
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph, stream=side):
                self.pre = self._run(chunks, kv_store)
        cur.wait_stream(side)
        self.pre_rope_k = dict(getattr(lw, "_pre_rope_k", {}) or {})
        self.logits = self.pre.logits
        self.idx = self.pre.idx

    def _run(self, chunks, kv_store):
        self.status.zero_()                          # each replay reports its own status bits
        return _selective_prefill(self.lw, chunks, kv_store, self.ratio, self.ck, self.mode, self.status,
                                  self.ids, extra_tokens=0, table=self.table, logits_rows=self.logits_rows,
                                  dense_logits=self.dense_logits)

    def replay(self, chunks: list[Chunk], kv_store: KVStore, input_ids: torch.Tensor | None = None):
        """Run the captured prefill for `chunks` (same lengths as the captured
        ones); returns the graph's static result (logits, idx, logits_sparse,
        fused_k / fused_v), valid until the next replay."""
        if [c.length for c in chunks] != self.lengths:
            raise ValueError(f"BlendGraph: chunk lengths {[c.length for c in chunks]} != captured {self.lengths}")
        with torch.inference_mode():
            entries = _store_entries(kv_store, chunks, "BlendGraph")
            sig = ops.chunk_signature(entries, self.table.layers)
            if sig != self._sig:                     # other tensors: point the table at them
                self.table.refresh(entries)
                self._sig = sig
            if input_ids is None:
                src = torch.tensor([[t for c in chunks for t in c.token_ids]], dtype=torch.int64)
                self.ids.copy_(src.pin_memory(), non_blocking=True)
            else:
                ids = input_ids.reshape(1, -1)
                if ids.shape[1] != self.S:
                    raise ValueError(f"input_ids has {ids.shape[1]} tokens, chunks have {self.S}")
                self.ids.copy_(ids, non_blocking=True)
            self.graph.replay()
        return self.pre

    def __call__(self, chunks: list[Chunk], kv_store: KVStore, input_ids: torch.Tensor | None = None):
        """Blended prefill of `chunks` (same lengths as the captured ones):
        logits (1, S, vocab) with rows outside the selection zero ((1, 1, vocab)
        for logits_rows "last"), in the graph's memory; the selection is in
        ``self.idx``.  ``input_ids`` (host -- preferably pinned -- or device)
        replaces the ids gathered from the chunks."""
        if not self.dense_logits:
            raise ValueError("BlendGraph(dense_logits=False) has no logits tensor: use replay()")
        return self.replay(chunks, kv_store, input_ids).logits
