"""cacheblend -- CacheBlend's selective-KV-recompute path on B200 (sm_100a).

Drop-in for the ``cacheblend`` package of cacheblend-hf-v7: the same public
names and signatures, with the hot path (chunk-KV concat + RoPE shift, HKVD
deviation + top-K, selective scatter, partial-query attention) running on
hand-written CUDA kernels in ``lib/libcbk.so`` (C ABI: include/cbk.h).
Importing the package loads the library; there is no CPU fallback.
"""
from __future__ import annotations

__version__ = "0.7.0+b200"

from cacheblend import _native  # noqa: F401  (loads libcbk.so or raises ImportError)
from cacheblend.tolerance import Tolerance, ToleranceResult, assert_logits_close
from cacheblend.model import LayerwiseModel, LayerwiseOutput
from cacheblend.kv_store import KVArena, KVStore
from cacheblend.chunker import Chunk, chunk_texts, fused_input_ids, chunk_offsets
from cacheblend.rope import apply_rope_shift
from cacheblend.precompute import precompute_chunk_kv, precompute_chunk_kv_into, precompute_from_cache_prompt
from cacheblend.fusor import fuse_full_recompute, fuse_full_reuse, fuse_selective, fuse_prefix_cache
from cacheblend.hkvd import kv_deviation, select_top_k
from cacheblend.generate import generate_greedy
from cacheblend.graph import BlendGraph

__all__ = [
    "Tolerance", "ToleranceResult", "assert_logits_close", "LayerwiseModel", "LayerwiseOutput",
    "KVStore", "KVArena", "Chunk", "chunk_texts", "fused_input_ids", "chunk_offsets", "apply_rope_shift",
    "precompute_chunk_kv", "precompute_chunk_kv_into", "precompute_from_cache_prompt", "fuse_full_recompute",
    "fuse_full_reuse", "fuse_selective", "fuse_prefix_cache", "kv_deviation", "select_top_k",
    "generate_greedy", "BlendGraph",
]
