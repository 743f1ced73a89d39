"""KVStore: chunk-level store of per-layer pre-RoPE K and V (API of
cacheblend-hf-v7 ``kv_store.py``): LRU at chunk granularity plus optional
background prefetch.

Entry layout: ``{"K": [Tensor(1, Lc, Hkv*D)] * n_layers, "V": [...]}``; the
blend kernels read these tensors in place through a pointer table, so they are
never copied into a staging buffer.
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
