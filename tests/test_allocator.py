"""Host-side page bookkeeping of the product pool (no GPU needed).

Re-runs the reference's known-answer allocator tests (tests/test_paged_cache.py,
tests/test_prefix_cache_eviction.py) on nano_vllm_b200's TinyKvPagedPool /
TinyKvPagedCache bookkeeping (``plan_append`` is the page logic of ``_append_chunk``
without the device write), and checks it step by step against the oracle's
restatement (oracle.PagePoolRef / PagedCacheRef) on random workloads.

The prefix-cache tests run the REFERENCE's own ``PrefixCache`` class, loaded from the
reference source tree, over the product pool: the drop-in claim is that the
reference's prefix cache needs nothing but these pools.  ``mlx.core`` is replaced by
a stub before loading (``PrefixCache`` never calls it; the module only names
``mx.array`` in type annotations).  They are skipped where the reference tree is
absent.
"""

import importlib.util
import os
import random
import sys
import types

import pytest

from nano_vllm_b200 import TinyKvPagedCache, TinyKvPagedPool

REF_PAGED = os.environ.get("NVM_REFERENCE_SRC", "/root/reference") + "/src/nano_vllm_metal/cache/paged.py"


def _reference_prefix_cache():
    """The reference's PrefixCache class (src/nano_vllm_metal/cache/paged.py:213-397)."""
    if not os.path.exists(REF_PAGED):
        pytest.skip("reference source tree not present")
    name = "_nvm_reference_cache"
    if name + ".paged" in sys.modules:
        return sys.modules[name + ".paged"].PrefixCache
    saved = {k: sys.modules.get(k) for k in ("mlx", "mlx.core")}
    mlx = types.ModuleType("mlx")
    core = types.ModuleType("mlx.core")
    core.array = type("array", (), {})
    mlx.core = core
    pkg = types.ModuleType(name)
    pkg.__path__ = []
    kv = types.ModuleType(name + ".kv_cache")
    kv.TinyKvCache = type("TinyKvCache", (), {})
    sys.modules.update({"mlx": mlx, "mlx.core": core, name: pkg, name + ".kv_cache": kv})
    try:
        spec = importlib.util.spec_from_file_location(name + ".paged", REF_PAGED)
        mod = importlib.util.module_from_spec(spec)
        sys.modules[name + ".paged"] = mod
        spec.loader.exec_module(mod)
    finally:
        for k, v in saved.items():
            if v is None:
                sys.modules.pop(k, None)
            else:
                sys.modules[k] = v
    return mod.PrefixCache


def PrefixCache(*args, **kwargs):  # noqa: N802 -- the reference's class, constructed over our pool
    return _reference_prefix_cache()(*args, **kwargs)


def test_paged_cache_page_counts():
    pool = TinyKvPagedPool(page_size=4)
    cache = TinyKvPagedCache(pool)
    total = 0
    for length in [3, 2, 5]:
        cache.plan_append(length)
        total += length
        assert cache.offset == total
        assert cache.num_pages == (total + 3) // 4
        assert sum(cache.page_lens) == total


def test_pool_reuses_freed_pages():
    pool = TinyKvPagedPool(page_size=4)
    first, second = TinyKvPagedCache(pool), TinyKvPagedCache(pool)
    first.plan_append(6)
    assert first.page_ids == [0, 1]
    assert pool.num_pages == 2 and pool.num_free_pages == 0
    first.release()
    assert first.offset == 0
    assert pool.num_pages == 2 and pool.num_free_pages == 2
    second.plan_append(5)
    assert pool.num_pages == 2 and pool.num_free_pages == 0
    assert set(second.page_ids) == {0, 1}


def test_rewind():
    pool = TinyKvPagedPool(page_size=4)
    cache = TinyKvPagedCache(pool)
    for length in [4, 3, 2]:
        cache.plan_append(length)
    assert cache.page_lens == [4, 4, 1]
    cache.rewind(3)
    assert cache.offset == 6
    assert cache.page_lens == [4, 2]
    assert cache.num_pages == 2
    assert pool.num_pages == 3 and pool.num_free_pages == 1


def test_layer_pools_are_independent():
    pools = [TinyKvPagedPool(page_size=4) for _ in range(2)]
    caches = [TinyKvPagedCache(p) for p in pools]
    for c in caches:
        c.plan_append(5)
    assert caches[0].page_ids == [0, 1] and caches[0].page_lens == [4, 1]
    assert caches[1].page_ids == caches[0].page_ids
    assert caches[0].page_ids is not caches[1].page_ids


def test_capacity_policy_matches_reference(oracle):
    """Geometric growth (paged.py:109-122) evaluated after every allocation."""
    pool, ref = TinyKvPagedPool(page_size=4), oracle.PagePoolRef(4)
    cache, rcache = TinyKvPagedCache(pool), oracle.PagedCacheRef(ref)
    for n in [3, 30, 1, 17, 60, 2, 90]:
        cache.plan_append(n)
        rcache.append_chunk(n)
        assert pool.capacity == ref.capacity
        assert cache.page_ids == rcache.page_ids and cache.page_lens == rcache.page_lens


@pytest.mark.parametrize("seed", range(4))
def test_random_workload_matches_oracle(oracle, seed):
    r = random.Random(seed)
    ps = r.choice([4, 16])
    pool, ref = TinyKvPagedPool(page_size=ps), oracle.PagePoolRef(ps)
    caches, rcaches = [], []
    for _ in range(300):
        op = r.random()
        if op < 0.3 or not caches:
            caches.append(TinyKvPagedCache(pool))
            rcaches.append(oracle.PagedCacheRef(ref))
        i = r.randrange(len(caches))
        if op < 0.7:
            n = r.randint(1, 3 * ps)
            assert caches[i].plan_append(n) == rcaches[i].append_chunk(n)
        elif op < 0.85:
            n = r.randint(0, caches[i].offset)
            caches[i].rewind(n)
            rcaches[i].rewind(n)
        else:
            caches[i].release()
            rcaches[i].release()
        assert caches[i].page_ids == rcaches[i].page_ids
        assert caches[i].page_lens == rcaches[i].page_lens
        assert pool.free_page_ids == ref.free_page_ids
        assert pool.ref_counts == ref.ref_counts
        assert pool.capacity == ref.capacity


def test_free_errors():
    pool = TinyKvPagedPool(page_size=4)
    pid = pool.allocate_page()
    pool.free_page(pid)
    with pytest.raises(ValueError):
        pool.free_page(pid)
    with pytest.raises(ValueError):
        pool.incref(pid)
    with pytest.raises(ValueError):
        TinyKvPagedPool(page_size=4, kv_bits=4)


# --- the reference's PrefixCache over the product pool
#     (reference tests/test_prefix_cache_eviction.py:8-90) -------------------------

def _run_request(pool, pc, num_layers, token_ids):
    caches = [TinyKvPagedCache(pool) for _ in range(num_layers)]
    matched = pc.match_prefix(token_ids)
    max_reuse = max(0, (len(token_ids) - 1) // pc.page_size)
    off = pc.attach(matched[:max_reuse], caches)
    while off < len(token_ids):
        n = min(pc.page_size, len(token_ids) - off)
        for c in caches:
            c.plan_append(n)
        off += n
    pc.register(token_ids, caches)
    for c in caches:
        c.release()
    return caches


def test_lru_eviction_bounds_cache_and_leaves_no_leak():
    pool = TinyKvPagedPool(page_size=4)
    pc = PrefixCache(pool, 2, max_blocks=3)
    for r in range(5):
        _run_request(pool, pc, 2, list(range(r * 100, r * 100 + 9)))
    assert pc.num_blocks <= 3
    assert pc.evicted_blocks > 0
    cached = {pid for e in pc.entries.values() for pid in e["pages"]}
    assert pool.used_page_ids == cached
    assert all(pool.ref_counts[p] == 1 for p in cached)
    pc.clear()
    assert pool.used_page_ids == set()
    assert pool.num_free_pages == pool.num_pages


def test_recently_used_prefix_survives_eviction():
    pool = TinyKvPagedPool(page_size=4)
    pc = PrefixCache(pool, 2, max_blocks=4)
    hot = list(range(9))
    _run_request(pool, pc, 2, hot)
    hot_hashes = pc.match_prefix(hot)
    assert len(hot_hashes) == 2
    for r in range(1, 6):
        pc.match_prefix(hot)
        _run_request(pool, pc, 2, list(range(r * 100, r * 100 + 9)))
    assert pc.match_prefix(hot) == hot_hashes
    assert pc.evicted_blocks > 0


def test_in_use_blocks_are_never_evicted():
    pool = TinyKvPagedPool(page_size=4)
    pc = PrefixCache(pool, 1, max_blocks=1)
    pinned = list(range(9))
    _run_request(pool, pc, 1, pinned)
    live = [TinyKvPagedCache(pool)]
    matched = pc.match_prefix(pinned)
    pc.attach(matched, live)
    for r in range(1, 5):
        _run_request(pool, pc, 1, list(range(r * 100, r * 100 + 9)))
    assert pc.match_prefix(pinned) == matched
    for c in live:
        c.release()


def test_prefix_attach_shares_pages():
    pool = TinyKvPagedPool(page_size=4)
    pc = PrefixCache(pool, 1)
    toks = list(range(10))
    _run_request(pool, pc, 1, toks)
    c = TinyKvPagedCache(pool)
    reused = pc.attach(pc.match_prefix(toks), [c])
    assert reused == 8 and c.page_lens == [4, 4] and c.offset == 8
    assert all(pool.ref_counts[p] == 2 for p in c.page_ids)
