"""KVStore: chunk-level store of per-layer pre-RoPE K and V (API of
cacheblend-hf-v7 ``kv_store.py``): LRU at chunk granularity plus optional
background prefetch.

Entry layout: ``{"K": [Tensor(1, Lc, Hkv*D)] * n_layers, "V": [...]}``; the
blend kernels read these tensors in place through a pointer table, so they are
never copied into a staging buffer.  ``KVArena`` keeps the same entries in one
pre-allocated device pool.
"""
from __future__ import annotations

from collections import OrderedDict
from concurrent.futures import Future, ThreadPoolExecutor
from typing import Callable, Optional

import torch

Entry = dict[str, list[torch.Tensor]]


class KVStore:
    def __init__(self, capacity: int = 1024, max_workers: int = 4):
        self.capacity = capacity
        self.max_workers = max_workers
        self._cache: "OrderedDict[str, Entry]" = OrderedDict()
        self._inflight: dict[str, Future] = {}
        self._executor: Optional[ThreadPoolExecutor] = None

    def has(self, chunk_id: str) -> bool:
        """True when the chunk is stored or being prefetched."""
        return chunk_id in self._cache or chunk_id in self._inflight

    def get(self, chunk_id: str) -> Entry:
        """Entry of a chunk (waits for an in-flight prefetch); marks it most recent."""
        fut = self._inflight.pop(chunk_id, None)
        if fut is not None:
            self._insert(chunk_id, fut.result())
        try:
            entry = self._cache[chunk_id]
        except KeyError:
            raise KeyError(f"KVStore miss: {chunk_id}") from None
        self._cache.move_to_end(chunk_id)
        return entry

    def put(self, chunk_id: str, K_per_layer: list[torch.Tensor], V_per_layer: list[torch.Tensor]) -> None:
        self._insert(chunk_id, {"K": K_per_layer, "V": V_per_layer})

    def _insert(self, chunk_id: str, entry: Entry) -> None:
        if chunk_id in self._cache:
            self._cache[chunk_id] = entry
            self._cache.move_to_end(chunk_id)
            return
        while len(self._cache) >= self.capacity:
            self.evict_lru()
        self._cache[chunk_id] = entry

    def evict_lru(self) -> Optional[str]:
        if not self._cache:
            return None
        cid, _ = self._cache.popitem(last=False)
        return cid

    def __len__(self) -> int:
        return len(self._cache)

    def clear(self) -> None:
        self._cache.clear()
        for fut in self._inflight.values():
            fut.cancel()
        self._inflight.clear()

    def prefetch_chunk(self, chunk_id: str, loader_fn: Callable[[], Entry]) -> Future:
        """Load a chunk in the background (idempotent); get() waits for it."""
        if chunk_id in self._cache:
            done: Future = Future()
            done.set_result(self._cache[chunk_id])
            return done
        if chunk_id in self._inflight:
            return self._inflight[chunk_id]
        if self._executor is None:
            self._executor = ThreadPoolExecutor(max_workers=self.max_workers,
                                                thread_name_prefix="kvstore-prefetch")
        fut = self._executor.submit(loader_fn)
        self._inflight[chunk_id] = fut
        return fut

    def shutdown(self, wait: bool = True) -> None:
        if self._executor is not None:
            self._executor.shutdown(wait=wait)
            self._executor = None


class KVArena(KVStore):
    """KVStore whose chunk K/V live in one pre-allocated device pool.

    Each chunk gets a contiguous slab of ``Lc`` token rows laid out
    ``[layer][K, V][Lc][kv_dim]``, so every per-layer tensor that ``get`` returns
    is a contiguous ``(1, Lc, kv_dim)`` view the blend kernels read in place, and
    ``put`` is one copy into the slab (no per-chunk allocations).  Slabs are
    placed first-fit in token units; when no free range is large enough the
    least recently used chunks are evicted until one is.  ``ops.ChunkTable``
    builds its pointer table for arena entries from the slab offsets in one
    vectorised step.  Same API and LRU semantics as KVStore.
    """

    def __init__(self, n_layers: int, kv_dim: int, capacity_tokens: int, device, dtype=torch.bfloat16,
                 capacity: int = 1024, max_workers: int = 4):
        super().__init__(capacity, max_workers)
        self.n_layers = int(n_layers)
        self.kv_dim = int(kv_dim)
        self.capacity_tokens = int(capacity_tokens)
        self.row_elems = self.n_layers * 2 * self.kv_dim          # elements per token row of a slab
        self.pool = torch.empty((self.capacity_tokens * self.row_elems,), dtype=dtype, device=device)
        self._free: list[list[int]] = [[0, self.capacity_tokens]]   # sorted [start, end) token ranges
        self._slab: dict[str, tuple[int, int]] = {}                 # chunk_id -> (start token, Lc)

    # -- allocation -----------------------------------------------------------
    def _alloc(self, n: int) -> Optional[int]:
        for r in self._free:
            if r[1] - r[0] >= n:
                start = r[0]
                r[0] += n
                if r[0] == r[1]:
                    self._free.remove(r)
                return start
        return None

    def _release(self, start: int, n: int) -> None:
        self._free.append([start, start + n])
        self._free.sort()
        merged: list[list[int]] = []
        for r in self._free:
            if merged and merged[-1][1] == r[0]:
                merged[-1][1] = r[1]
            else:
                merged.append(r)
        self._free = merged

    def free_tokens(self) -> int:
        return sum(e - s for s, e in self._free)

    def _views(self, start: int, n: int) -> Entry:
        slab = self.pool[start * self.row_elems:(start + n) * self.row_elems].view(self.n_layers, 2, n, self.kv_dim)
        # "_slab": (pool address, first token, tokens, elements per token row, layers, kv_dim)
        return {"K": [slab[l, 0].unsqueeze(0) for l in range(self.n_layers)],
                "V": [slab[l, 1].unsqueeze(0) for l in range(self.n_layers)],
                "_slab": (self.pool.data_ptr(), start, n, self.row_elems, self.n_layers, self.kv_dim)}

    def reserve(self, chunk_id: str, n_tokens: int) -> Entry:
        """Slab for a chunk of n_tokens (evicting LRU chunks as needed); returns its
        entry so a producer can write the K/V in place.  Replaces an existing entry."""
        if n_tokens <= 0 or n_tokens > self.capacity_tokens:
            raise ValueError(f"KVArena: chunk of {n_tokens} tokens does not fit {self.capacity_tokens}")
        if chunk_id in self._cache:
            self._drop(chunk_id)
        start = self._alloc(n_tokens)
        while start is None:
            if self.evict_lru() is None:
                raise MemoryError("KVArena: no free range after evicting every chunk")
            start = self._alloc(n_tokens)
        while len(self._cache) >= self.capacity:
            self.evict_lru()
        entry = self._views(start, n_tokens)
        self._slab[chunk_id] = (start, n_tokens)
        self._cache[chunk_id] = entry
        return entry

    # -- KVStore API ------------------------------------------------------------
    def put(self, chunk_id: str, K_per_layer: list[torch.Tensor], V_per_layer: list[torch.Tensor]) -> None:
        if len(K_per_layer) != self.n_layers or len(V_per_layer) != self.n_layers:
            raise ValueError(f"KVArena: expected {self.n_layers} layers")
        n = K_per_layer[0].shape[-2]
        entry = self.reserve(chunk_id, n)
        with torch.no_grad():
            for l in range(self.n_layers):
                entry["K"][l].copy_(K_per_layer[l].reshape(1, n, self.kv_dim))
                entry["V"][l].copy_(V_per_layer[l].reshape(1, n, self.kv_dim))

    def _insert(self, chunk_id: str, entry: Entry) -> None:
        # prefetched entries (loader output) are copied into the pool
        slab = entry.get("_slab")
        if slab is not None and slab[0] == self.pool.data_ptr() and self._slab.get(chunk_id) == slab[1:3]:
            self._cache[chunk_id] = entry
            self._cache.move_to_end(chunk_id)
            return
        self.put(chunk_id, entry["K"], entry["V"])

    def _drop(self, chunk_id: str) -> None:
        self._cache.pop(chunk_id, None)
        slab = self._slab.pop(chunk_id, None)
        if slab is not None:
            self._release(*slab)

    def evict_lru(self) -> Optional[str]:
        if not self._cache:
            return None
        cid = next(iter(self._cache))
        self._drop(cid)
        return cid

    def clear(self) -> None:
        super().clear()
        self._slab.clear()
        self._free = [[0, self.capacity_tokens]]
