"""Device-side page allocation (nvm_paged_append) vs the reference's sequential semantics."""

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
    with pytest.raises(RuntimeError, match="allocate_page"):
        dt.check_status()
    assert torch.equal(dt.block_table, before[0]) and torch.equal(dt.context_lens, before[1])
    assert torch.equal(dt.num_pages, before[2])
