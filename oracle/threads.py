"""Host-core parallelism for the oracle's fp32 model replay -- test
infrastructure and the timed CPU baseline.

numpy runs elementwise ufuncs on one core and releases the GIL inside them and
inside BLAS calls, so independent pieces of work (attention heads, blocks of
rows) run concurrently from a thread pool.  While the pool works, BLAS is
limited to one thread per call so the pool's threads do not oversubscribe the
cores; large GEMMs outside the pool keep BLAS's own threading.
"""
from __future__ import annotations

import os
from concurrent.futures import ThreadPoolExecutor
from contextlib import contextmanager

_POOL = None


def n_threads() -> int:
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except AttributeError:
        return max(1, os.cpu_count() or 1)


def pool() -> ThreadPoolExecutor:
    global _POOL
    if _POOL is None:
        _POOL = ThreadPoolExecutor(max_workers=n_threads(), thread_name_prefix="oracle")
    return _POOL


@contextmanager
def single_threaded_blas():
    try:
        from threadpoolctl import threadpool_limits
    except ImportError:
        yield
        return
    with threadpool_limits(limits=1, user_api="blas"):
        yield


def run(tasks):
    """Run zero-argument callables on the pool (BLAS single-threaded meanwhile)
    and return their results in order."""
    tasks = list(tasks)
    if len(tasks) <= 1 or n_threads() == 1:
        return [t() for t in tasks]
    with single_threaded_blas():
        futs = [pool().submit(t) for t in tasks]
        return [f.result() for f in futs]


def row_chunks(n: int, min_rows: int = 64):
    """[start, end) row ranges splitting n rows over the pool's threads."""
    parts = max(1, min(n_threads(), n // min_rows))
    step = -(-n // parts)
    return [(a, min(n, a + step)) for a in range(0, n, step)]
