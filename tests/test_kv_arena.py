"""KVArena: the KVStore API over one pre-allocated pool (slab allocation,
LRU eviction by tokens, views that alias the pool).  CPU pool here; the GPU
tests check the kernels read arena entries identically to plain entries."""
import pytest
import torch


def _arena(cap_tokens=100, layers=3, kv=8, capacity=1024):
    from cacheblend import KVArena
    return KVArena(layers, kv, cap_tokens, torch.device("cpu"), dtype=torch.float32, capacity=capacity)


def _kv(n, layers=3, kv=8, seed=0):
    g = torch.Generator().manual_seed(seed)
    return ([torch.randn((1, n, kv), generator=g) for _ in range(layers)],
            [torch.randn((1, n, kv), generator=g) for _ in range(layers)])


def test_put_get_round_trip_and_views_alias_pool():
    a = _arena()
    K, V = _kv(10)
    a.put("c0", K, V)
    e = a.get("c0")
    for l in range(3):
        assert torch.equal(e["K"][l], K[l]) and torch.equal(e["V"][l], V[l])
        assert e["K"][l].shape == (1, 10, 8) and e["K"][l].is_contiguous()
        assert e["K"][l].untyped_storage().data_ptr() == a.pool.untyped_storage().data_ptr()
    assert a.free_tokens() == 90 and len(a) == 1 and a.has("c0")


def test_eviction_by_tokens_is_lru():
    a = _arena(cap_tokens=30)
    for i in range(3):
        a.put(f"c{i}", *_kv(10, seed=i))
    a.get("c0")                                  # c1 becomes least recent
    a.put("c3", *_kv(10, seed=3))
    assert not a.has("c1") and a.has("c0") and a.has("c2") and a.has("c3")
    with pytest.raises(KeyError):
        a.get("c1")
    e0 = a.get("c0")
    assert torch.equal(e0["K"][2], _kv(10, seed=0)[0][2])   # surviving data untouched


def test_fragmentation_evicts_until_a_range_fits():
    a = _arena(cap_tokens=40)
    for i in range(4):
        a.put(f"c{i}", *_kv(10, seed=i))
    a._drop("c1")                                # holes: [10,20)
    a.put("big", *_kv(20, seed=9))               # needs 20 contiguous: evicts LRU c0 -> [0,20)
    assert a.has("big") and not a.has("c0") and a.has("c2") and a.has("c3")
    assert torch.equal(a.get("big")["V"][1], _kv(20, seed=9)[1][1])
    assert a.free_tokens() == 0


def test_capacity_in_chunks_and_replace_and_clear():
    a = _arena(cap_tokens=100, capacity=2)
    a.put("a", *_kv(5, seed=1))
    a.put("b", *_kv(5, seed=2))
    a.put("c", *_kv(5, seed=3))                  # chunk-count capacity evicts "a"
    assert not a.has("a") and len(a) == 2
    a.put("b", *_kv(7, seed=4))                  # replace: old slab freed, new one used
    assert a.get("b")["K"][0].shape == (1, 7, 8) and a.free_tokens() == 100 - 12
    a.clear()
    assert len(a) == 0 and a.free_tokens() == 100
    with pytest.raises(ValueError):
        a.put("x", *_kv(5, layers=2))
    with pytest.raises(ValueError):
        a.reserve("y", 101)


def test_prefetch_into_arena():
    a = _arena()
    K, V = _kv(6, seed=5)
    fut = a.prefetch_chunk("p", lambda: {"K": K, "V": V})
    fut.result()
    e = a.get("p")
    assert torch.equal(e["K"][1], K[1]) and "_slab" in e
    a.shutdown()
