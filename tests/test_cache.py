"""Expert-cache bookkeeping (qmoe_cache_*, csrc/qmoe_cache.c) against the
cases of the reference's c/tests/test_cache.c. Host-only: no GPU needed."""
import ctypes as C
import threading

import pytest


@pytest.fixture
def L(built):
    import qmoe
    return qmoe.lib()


class Cache:
    def __init__(self, L, budget, policy, parts=0):
        self.L = L
        self.h = L.qmoe_cache_new(budget, policy, parts)

    def put(self, key, val, nbytes, pin=0, hot=0):
        ev = (C.c_uint64 * 64)()
        n = C.c_size_t()
        ok = self.L.qmoe_cache_put(self.h, key, val, nbytes, pin, hot, ev, 64, C.byref(n))
        self.last_evicted = [ev[i] for i in range(min(n.value, 64))]
        return ok

    def peek(self, key):
        v = C.c_uint64()
        return v.value if self.L.qmoe_cache_peek(self.h, key, C.byref(v)) else None

    def get(self, key):
        v = C.c_uint64()
        return v.value if self.L.qmoe_cache_get(self.h, key, C.byref(v)) else None

    def stats(self):
        return self.L.qmoe_cache_stats_get(self.h).as_dict()

    def close(self):
        self.L.qmoe_cache_free(self.h)


LRU, LFU, ADAPTIVE = 0, 1, 2


def test_basic(L):
    c = Cache(L, 1000, LRU)
    assert c.put(1, 11, 100) == 1 and c.put(2, 12, 100) == 1
    assert c.peek(1) == 11 and c.get(2) == 12 and c.get(3) is None
    s = c.stats()
    assert s["hits"] == 1 and s["misses"] == 1 and s["size"] == 2 and s["bytes"] == 200
    c.close()


def test_lru(L):
    c = Cache(L, 300, LRU)
    for k in (1, 2, 3):
        assert c.put(k, k, 100)
    assert c.get(1) == 1          # 2 becomes the oldest
    assert c.put(4, 4, 100)
    assert c.last_evicted == [2]
    assert c.peek(2) is None and c.peek(1) and c.peek(3) and c.peek(4)
    c.close()


def test_lfu(L):
    c = Cache(L, 300, LFU)
    for k in (1, 2, 3):
        c.put(k, k, 100)
    c.get(1); c.get(1); c.get(2)
    assert c.put(4, 4, 100)
    assert c.peek(3) is None and c.peek(1) and c.peek(2)
    c.close()


def test_adaptive(L):
    c = Cache(L, 300, ADAPTIVE)
    assert c.put(1, 1, 100, hot=1)
    assert c.put(2, 2, 200)
    assert c.put(3, 3, 100)
    assert c.peek(2) is None and c.peek(1) and c.peek(3)
    c.close()


def test_pin(L):
    c = Cache(L, 200, LRU)
    assert c.put(1, 1, 100, pin=1)
    assert c.put(2, 2, 100)
    assert L.qmoe_cache_pin(c.h, 2) == 1
    assert c.put(3, 3, 100) == 0
    assert c.peek(1) and c.peek(2) and c.peek(3) is None
    assert L.qmoe_cache_unpin(c.h, 2) == 1
    assert c.put(3, 3, 100) == 1
    assert c.peek(1) and c.peek(2) is None and c.peek(3)
    s = c.stats()
    assert s["pinned"] == 1 and s["rejected"] == 1
    c.close()


def test_hot_retained(L):
    c = Cache(L, 200, LRU)
    assert c.put(1, 1, 100, hot=1)
    assert c.put(2, 2, 100)
    assert c.put(3, 3, 100)
    assert c.peek(1) and c.peek(2) is None and c.peek(3)
    c.close()


def test_partitions(L):
    c = Cache(L, 200, LRU, 2)
    assert c.put(0x100000001, 1, 100) and c.put(0x100000002, 2, 100)
    assert c.put(0x200000001, 3, 100)     # partition 1 is over its share: it pays
    assert c.last_evicted == [1]
    assert c.put(0x200000002, 4, 100)
    assert c.peek(0x100000001) is None or c.peek(0x100000002) is None
    assert c.peek(0x200000001) and c.peek(0x200000002)
    c.close()


def test_partition_over_share_pays_first(L):
    c = Cache(L, 400, LRU, 2)
    for i in (1, 2, 3):
        assert c.put(0x100000000 + i, i, 100)   # partition 1: 300 > fair 200
    assert c.put(0x200000001, 4, 100)
    assert c.put(0x200000002, 5, 100)            # evicts partition 1's LRU
    assert c.last_evicted == [1]
    assert c.peek(0x200000001) and c.peek(0x200000002)
    c.close()


def test_replace_keeps_pin(L):
    c = Cache(L, 300, LRU)
    assert c.put(1, 1, 100, pin=1)
    assert c.put(1, 9, 100)
    assert c.peek(1) == 9
    s = c.stats()
    assert s["pinned"] == 1 and s["size"] == 1 and s["bytes"] == 100
    c.close()


def test_oversized(L):
    c = Cache(L, 100, LRU)
    assert c.put(1, 1, 200) == 0
    assert c.put(2, 2, 50) == 1
    assert c.put(3, 3, 100) == 1
    assert c.peek(2) is None
    c.close()


def test_table_stress_and_erase(L):
    n = 5000
    c = Cache(L, 0, LRU)
    keys = [(i * 0x9E3779B97F4A7C15) & 0xFFFFFFFFFFFF for i in range(n)]
    for k in keys:
        assert c.put(k, k & 0xFFFF, 1)
    for k in keys:
        assert c.peek(k) == k & 0xFFFF
    v = C.c_uint64()
    for k in keys[: n // 2]:
        assert L.qmoe_cache_erase(c.h, k, C.byref(v)) == 1
    s = c.stats()
    assert s["size"] == n // 2 and s["bytes"] == n // 2
    for i, k in enumerate(keys):
        assert (c.peek(k) is None) == (i < n // 2)
    c.close()


def test_concurrent_bytes_within_budget(L):
    """8 threads hammering put/get never exceed the budget (test_cache.c:198-218)."""
    c = Cache(L, 64 * 100, ADAPTIVE, 4)
    errors = []

    def worker(tid):
        try:
            ev = (C.c_uint64 * 64)()
            n = C.c_size_t()
            v = C.c_uint64()
            for i in range(2000):
                key = ((tid % 4) << 32) | ((i * 7 + tid) % 97)
                L.qmoe_cache_put(c.h, key, i, 100, 0, i % 5 == 0, ev, 64, C.byref(n))
                L.qmoe_cache_get(c.h, key ^ 1, C.byref(v))
        except Exception as e:  # pragma: no cover
            errors.append(e)

    ts = [threading.Thread(target=worker, args=(t,)) for t in range(8)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    s = c.stats()
    assert not errors
    assert s["bytes"] <= 64 * 100 and s["peak_bytes"] <= 64 * 100
    c.close()


def test_rejected_put_reports_the_victims_it_dropped(L):
    """cache.c:236-242: a put that runs out of unpinned victims is rejected,
    and the victims it had already dropped stay out (no rollback); it reports
    them, so the pool can free their slots."""
    c = Cache(L, 300, LRU)
    assert c.put(1, 11, 100) and c.put(2, 22, 100, pin=1) and c.put(3, 33, 100, pin=1)
    assert c.put(4, 44, 200) == 0
    assert c.last_evicted == [11]
    assert c.peek(1) is None and c.peek(2) == 22 and c.peek(3) == 33 and c.peek(4) is None
    s = c.stats()
    assert s["rejected"] == 1 and s["evictions"] == 0 and s["bytes"] == 200 and s["size"] == 2
    assert c.put(4, 44, 100) == 1          # the freed room is usable
    c.close()


def test_rejected_replacement_preserves_existing_value(L):
    """tests/test_cache.py:32-41 of the reference: an oversized replacement is
    refused before the old entry is touched."""
    c = Cache(L, 2, LRU)
    assert c.put(7, 1, 2)
    assert c.put(7, 2, 3) == 0
    assert c.get(7) == 1
    s = c.stats()
    assert s["rejected"] == 1 and s["evictions"] == 0 and s["bytes"] == 2
    c.close()


def test_eviction_and_pinning_of_the_python_runtime(L):
    """tests/test_cache.py:6-16 of the reference (ExpertCache(max_items=2));
    the item limit is a byte budget here, one byte per item."""
    c = Cache(L, 2, LRU)
    assert c.put(1, 1, 1) and c.put(2, 2, 1, pin=1) and c.put(3, 3, 1)
    assert c.get(1) is None and c.get(2) == 2 and c.get(3) == 3
    s = c.stats()
    assert s["evictions"] >= 1 and s["pinned"] == 1
    c.close()


def test_partition_over_its_share_of_the_python_runtime(L):
    """tests/test_cache.py:19-29 of the reference: with two layer partitions,
    the layer over its fair share gives up its oldest entry."""
    c = Cache(L, 4, ADAPTIVE, parts=2)
    k = lambda layer, e: (layer << 32) | e
    for key in (k(0, 0), k(0, 1), k(0, 2), k(1, 0), k(1, 1)):
        assert c.put(key, key + 1, 1)
    assert c.peek(k(0, 0)) is None
    assert c.peek(k(1, 0)) == k(1, 0) + 1 and c.peek(k(1, 1)) == k(1, 1) + 1
    # partition bytes {0: 2, 1: 2}
    assert c.peek(k(0, 1)) is not None and c.peek(k(0, 2)) is not None
    assert c.stats()["bytes"] == 4
    c.close()
