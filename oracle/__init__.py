"""CPU oracle for CacheBlend's selective-KV-recompute path -- TEST INFRASTRUCTURE.

This package restates, in numpy, the algorithm of the reference implementation
(cacheblend-hf-v7, ``src/cacheblend``) for the hot path: chunk-KV concat,
RoPE shift, HKVD deviation + top-K, the force-include rule, the selective
scatter, partial-query attention and the whole ``fuse_selective`` forward of a
Mistral/Llama-style decoder.  Every function cites the reference file:line it
follows.

Parity is pinned: ``tests/test_oracle_golden.py`` checks these functions
against golden vectors produced by running the reference itself
(``tests/golden/make_golden.py``).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
reference arm may import this package, and only as the checker or the timed
CPU baseline.  The product (``cacheblend-hf-v7_b200/cacheblend``) never imports it.
"""
from oracle.bf16 import bf16_to_f32, f32_to_bf16, round_bf16  # noqa: F401
from oracle import hotpath, model  # noqa: F401
