"""Device-side batch metadata (nvm_paged_append / nvm_paged_rewind / nvm_paged_attach) vs the
reference's sequential semantics (TinyKvPagedCache._append_chunk, rewind, release,
PrefixCache.attach over one TinyKvPagedPool), restated in oracle.PagePoolRef / PagedCacheRef."""

import random

import pytest
import torch

from nano_vllm_b200 import DevicePageTable

pytestmark = pytest.mark.gpu


def _simulate(oracle, steps, B, ps, prefree):
    """Reference semantics: per step, for b in order, PagedCacheRef.append_chunk(new[b])."""
    pool = oracle.PagePoolRef(ps)
    for _ in range(prefree):
        pool.allocate_page()
    held = list(range(prefree))
    random.Random(0).shuffle(held)
    for pid in held:
        pool.free_page(pid)  # free list in a scrambled LIFO order
    caches = [oracle.PagedCacheRef(pool) for _ in range(B)]
    slots_per_step = []
    for new in steps:
        s = []
        for b in range(B):
            if new[b] > 0:
                s += caches[b].append_chunk(new[b])
        slots_per_step.append(s)
    return pool, caches, slots_per_step, held


@pytest.mark.parametrize("ps", [4, 16])
def test_append_matches_sequential_reference(cuda, oracle, ps):
    r = random.Random(ps)
    B, MP, cap = 7, 64, 400
    steps = [[r.choice([0, 1, 1, 2, ps, 3 * ps + 1]) for _ in range(B)] for _ in range(6)]
    pool, caches, ref_slots, held = _simulate(oracle, steps, B, ps, prefree=10)
    dt = DevicePageTable(B, MP, ps, cap)
    # same starting pool: ids 0..9 minted, all free, in the same LIFO order
    dt.free_stack[:10] = torch.tensor(held, dtype=torch.int32)  # free_stack[top-1] is popped first
    dt.free_top.fill_(10)
    dt.num_pages.fill_(10)
    for i, new in enumerate(steps):
        slots = dt.append(torch.tensor(new, dtype=torch.int32))
        dt.check_status()
        assert slots.tolist() == ref_slots[i]
    for b in range(B):
        row = dt.block_table[b].tolist()
        assert row[:caches[b].num_pages] == caches[b].page_ids
        assert all(x == -1 for x in row[caches[b].num_pages:])
    assert dt.context_lens.tolist() == [c.offset for c in caches]
    assert int(dt.num_pages.item()) == pool.num_pages
    assert int(dt.free_top.item()) == len(pool.free_page_ids)
    rc = dt.refcount.tolist()
    for pid in pool.used_page_ids:
        assert rc[pid] == 1


def test_out_of_pages_writes_nothing(cuda):
    dt = DevicePageTable(2, 4, 16, 3)
    dt.append(torch.tensor([16, 16], dtype=torch.int32))
    dt.check_status()
    before = (dt.block_table.clone(), dt.context_lens.clone(), dt.num_pages.clone())
    dt.append(torch.tensor([40, 1], dtype=torch.int32), slot_mapping=torch.empty(41, dtype=torch.int64,
                                                                                   device="cuda"))
    with pytest.raises(RuntimeError, match="device call failed"):
        dt.check_status()
    assert torch.equal(dt.block_table, before[0]) and torch.equal(dt.context_lens, before[1])
    assert torch.equal(dt.num_pages, before[2])


def _compare(dt, pool, caches):
    """Device tables == the oracle's bookkeeping (rows, lengths, LIFO order, refcounts)."""
    B = len(caches)
    for b in range(B):
        row = dt.block_table[b].tolist()
        assert row[:caches[b].num_pages] == caches[b].page_ids, b
        assert all(x == -1 for x in row[caches[b].num_pages:]), b
    assert dt.context_lens.tolist() == [c.offset for c in caches]
    assert dt.free_list() == pool.free_page_ids
    assert int(dt.num_pages.item()) == pool.num_pages
    rc = dt.refcount.tolist()
    for pid in range(pool.num_pages):
        assert rc[pid] == pool.ref_counts.get(pid, 0), pid
    assert all(x == -1 for x in dt.last_call.tolist())


@pytest.mark.parametrize("seed", [0, 1, 2])
def test_append_attach_rewind_release_sequence(cuda, oracle, seed):
    """A serving trace: prompts, a prefix shared through the index, speculative-verify
    rewinds of rejected draft tokens, request completion, page reuse."""
    r = random.Random(seed)
    B, MP, ps, cap = 6, 32, 4, 256
    pool = oracle.PagePoolRef(ps)
    caches = [oracle.PagedCacheRef(pool) for _ in range(B)]
    dt = DevicePageTable(B, MP, ps, cap)

    def append(new):
        ref = []
        for b in range(B):
            if new[b] > 0:
                ref += caches[b].append_chunk(new[b])
        slots = dt.append(torch.tensor(new, dtype=torch.int32))
        dt.check_status()
        assert slots.tolist() == ref
        _compare(dt, pool, caches)

    def rewind(n):
        for b in range(B):
            caches[b].rewind(n[b])
        dt.rewind(torch.tensor(n, dtype=torch.int32))
        dt.check_status()
        _compare(dt, pool, caches)

    # prompts for requests 0..2
    append([r.randint(9, 23), r.randint(1, 12), r.randint(4, 30), 0, 0, 0])
    # the prefix index registers request 0's first two full pages (it owns a reference)
    shared = caches[0].page_ids[:2]
    for pid in shared:
        pool.incref(pid)
    dt.refcount[torch.tensor(shared, device="cuda").long()] += 1
    # requests 3 and 4 attach that prefix
    for b in (3, 4):
        caches[b].attach(shared)
    pages = torch.full((B, 4), -1, dtype=torch.int32)
    pages[3, :2] = torch.tensor(shared)
    pages[4, :2] = torch.tensor(shared)
    dt.attach(pages, torch.tensor([0, 0, 0, 2, 2, 0], dtype=torch.int32))
    dt.check_status()
    _compare(dt, pool, caches)
    # decode / verify rounds: append k+1 tokens, keep a random prefix of them
    for _ in range(4):
        new = [r.choice([0, 1, 5]) for _ in range(B)]
        append(new)
        rewind([r.randint(0, new[b]) if new[b] else 0 for b in range(B)])
    # a long rewind into shared pages, a full release through rewind, then release()
    n = [0] * B
    n[4] = caches[4].offset - 1
    n[1] = caches[1].offset
    rewind(n)
    mask = torch.zeros(B, dtype=torch.bool)
    mask[0] = True
    mask[3] = True
    for b in (0, 3):
        caches[b].release()
    dt.release(mask)
    dt.check_status()
    _compare(dt, pool, caches)
    # freed pages come back LIFO
    append([ps + 1, 2, 0, 3 * ps, 1, 7])


def test_invalid_rewind_and_attach_write_nothing(cuda):
    dt = DevicePageTable(3, 8, 4, 32)
    dt.append(torch.tensor([5, 9, 0], dtype=torch.int32))
    dt.check_status()
    snap = [t.clone() for t in (dt.block_table, dt.context_lens, dt.refcount, dt.free_stack, dt.free_top)]
    dt.rewind(torch.tensor([1, 10, 0], dtype=torch.int32))  # 10 > length 9
    with pytest.raises(RuntimeError, match="device call failed"):
        dt.check_status()
    for a, b in zip(snap, (dt.block_table, dt.context_lens, dt.refcount, dt.free_stack, dt.free_top)):
        assert torch.equal(a, b)
    pages = torch.tensor([[0, -1], [0, -1], [0, -1]], dtype=torch.int32)
    dt.attach(pages, torch.tensor([1, 0, 0], dtype=torch.int32))  # request 0 is not fresh
    with pytest.raises(RuntimeError, match="device call failed"):
        dt.check_status()
    for a, b in zip(snap, (dt.block_table, dt.context_lens, dt.refcount, dt.free_stack, dt.free_top)):
        assert torch.equal(a, b)


def test_rewind_many_requests_shared_pages(cuda, oracle):
    """Thousands of calls across the CTA: two prefix pages shared by every request return
    to the free list exactly once, at the call that drops their last reference."""
    B, MP, ps, cap = 1500, 8, 16, 8192
    pool = oracle.PagePoolRef(ps)
    caches = [oracle.PagedCacheRef(pool) for _ in range(B)]
    dt = DevicePageTable(B, MP, ps, cap)
    first = [2 * ps] + [0] * (B - 1)
    ref = caches[0].append_chunk(2 * ps)
    assert dt.append(torch.tensor(first, dtype=torch.int32)).tolist() == ref
    shared = caches[0].page_ids[:2]
    for b in range(1, B):
        caches[b].attach(shared)
    pages = torch.full((B, 2), -1, dtype=torch.int32)
    pages[1:] = torch.tensor(shared, dtype=torch.int32)
    dt.attach(pages, torch.tensor([0] + [2] * (B - 1), dtype=torch.int32))
    dt.check_status()
    new = [1 + (b * 7) % 40 for b in range(B)]
    ref = []
    for b in range(B):
        ref += caches[b].append_chunk(new[b])
    assert dt.append(torch.tensor(new, dtype=torch.int32)).tolist() == ref
    dt.check_status()
    _compare(dt, pool, caches)
    n = [caches[b].offset if b % 3 == 0 else (b % 5) for b in range(B)]
    for b in range(B):
        caches[b].rewind(n[b])
    dt.rewind(torch.tensor(n, dtype=torch.int32))
    dt.check_status()
    _compare(dt, pool, caches)
    # everyone left releases: the shared pages go back once, after their last owner
    for b in range(B):
        caches[b].release()
    dt.release()
    dt.check_status()
    _compare(dt, pool, caches)
