"""Multi-rank host logic on CPU (gloo, world sizes 2 and 4): the KV-head-sharded
HKVD exchange and failure detection by a short process-group timeout."""
import os
import socket
import time

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from oracle import hotpath as hp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _init(rank, world, port, timeout_s=60):
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))
    return dist


def _data(S=3000, n_kv=8, D=16, seed=0):
    rng = np.random.default_rng(seed)
    old = rng.standard_normal((S, n_kv * D)).astype(np.float32)
    new = old + (rng.random((S, 1)) < 0.2) * rng.standard_normal((S, n_kv * D)).astype(np.float32) * 0.05
    return new.astype(np.float32), old


def _sharded_worker(rank, world, port, out):
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                    "cacheblend-hf-v7_b200"))
    from cacheblend.sharding import exchange_deviation, head_shard
    dist = _init(rank, world, port)
    new, old = _data()
    n_kv, D = 8, 16
    lo, hi = head_shard(n_kv, world, rank)
    cols = slice(lo * D, hi * D)
    partial = torch.from_numpy(hp.kv_deviation(new[:, cols], old[:, cols]))
    total = exchange_deviation(partial)
    k = hp.topk_count(len(new), 0.15)
    idx = hp.topk_select(total.numpy(), k, force_last=True)
    out[rank] = (total.numpy().tobytes(), idx.tobytes())
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_head_sharded_hkvd_exchange_identical_on_all_ranks(world):
    """Every rank ends with the same deviations and selection, and they are
    the single-device ones bit for bit (each rank's heads are a subtree of the
    deviation's pairwise tree, and the exchange combines with the same tree)."""
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    port = _free_port()
    mp.start_processes(_sharded_worker, args=(world, port, out), nprocs=world, join=True,
                       start_method="spawn")
    for r in range(1, world):
        assert out[r] == out[0]                          # same bits on every rank
    t0, i0 = out[0]
    new, old = _data()
    single_dev = hp.kv_deviation(new, old)
    np.testing.assert_array_equal(np.frombuffer(t0, np.float32), single_dev)
    single = hp.topk_select(single_dev, hp.topk_count(len(new), 0.15), force_last=True)
    np.testing.assert_array_equal(np.frombuffer(i0, np.int64), single)


def _failing_worker(rank, world, port, out):
    dist = _init(rank, world, port, timeout_s=3)
    if rank == 1:
        out[1] = "left"        # leaves between steps, no collective in flight
        return
    t = time.time()
    try:
        dist.all_reduce(torch.ones(4))
        out[0] = "no error"
    except Exception as e:    # the short PG timeout ends the collective with an error
        out[0] = f"error after {time.time() - t:.1f}s: {type(e).__name__}"


def test_rank_failure_is_detected_by_timeout():
    world = 2
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    ctx = mp.start_processes(_failing_worker, args=(world, _free_port(), out), nprocs=world,
                             join=False, start_method="spawn")
    deadline = time.time() + 60
    while time.time() < deadline and 0 not in out:
        time.sleep(0.2)
    for p in ctx.processes:
        p.join(timeout=10)
        if p.is_alive():
            p.kill()
    assert out.get(1) == "left"
    assert str(out.get(0, "")).startswith("error"), out.get(0)


@pytest.mark.parametrize("n_kv,world", [(8, 1), (8, 2), (8, 4), (8, 8)])
def test_head_shard_ranges(n_kv, world):
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                    "cacheblend-hf-v7_b200"))
    from cacheblend.sharding import head_shard
    spans = [head_shard(n_kv, world, r) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == n_kv
    assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    with pytest.raises(ValueError):
        head_shard(8, 3, 0)
