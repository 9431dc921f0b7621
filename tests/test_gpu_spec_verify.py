"""Batched speculative-decoding acceptance on the device against the reference's
per-request loop (engine/generate.py:130-169, restated by oracle.spec_accept_ref), and
the verify step's page-table update (one batched rewind) against the sequential
rewind / release of the reference's caches (oracle.PagedCacheRef)."""

import numpy as np
import pytest
import torch

from nano_vllm_b200 import DevicePageTable, verify_accept

pytestmark = pytest.mark.gpu


def _random_batch(rng, B, K1, vocab):
    cand = rng.integers(0, vocab, (B, K1))
    ver = rng.integers(0, vocab, (B, K1))
    # make long accepted runs common: the first cut[b] drafts are what the target predicts
    cut = rng.integers(0, K1, B)
    for b in range(B):
        ver[b, :cut[b]] = cand[b, 1:cut[b] + 1]
    return cand.astype(np.int32), ver.astype(np.int32)


@pytest.mark.parametrize("K1", [1, 2, 5, 9])
@pytest.mark.parametrize("eos", [None, 3])
@pytest.mark.parametrize("with_budget", [False, True])
def test_accept_matches_sequential_loop(cuda, oracle, K1, eos, with_budget):
    rng = np.random.default_rng(K1 * 10 + (eos or 0) + with_budget)
    B = 777
    cand, ver = _random_batch(rng, B, K1, 6)
    budget = rng.integers(-1, K1 + 2, B).astype(np.int32) if with_budget else None
    active = (rng.random(B) > 0.1).astype(np.int32)
    res = verify_accept(torch.from_numpy(cand).to(cuda), torch.from_numpy(ver).to(cuda), eos_id=eos,
                        budget=None if budget is None else torch.from_numpy(budget).to(cuda),
                        active=torch.from_numpy(active).to(cuda))
    got = {k: v.cpu().numpy() for k, v in res._asdict().items()}
    for b in range(B):
        if not active[b]:
            assert got["n_emitted"][b] == 0 and got["rewind"][b] == 0 and not got["finished"][b]
            assert got["next_token"][b] == -1 and (got["emitted"][b] == -1).all()
            continue
        lim = None if budget is None or budget[b] < 0 else int(budget[b])
        emitted, nxt, rw, drw, fin = oracle.spec_accept_ref(cand[b].tolist(), ver[b].tolist(), eos, lim)
        n = len(emitted)
        assert got["n_emitted"][b] == n, b
        assert got["emitted"][b, :n].tolist() == emitted and (got["emitted"][b, n:] == -1).all(), b
        assert got["next_token"][b] == (-1 if nxt is None else nxt), b
        assert (got["rewind"][b], got["draft_rewind"][b], bool(got["finished"][b])) == (rw, drw, fin), b


def test_verify_step_page_tables(cuda, oracle):
    """Append K1 candidate tokens per request, accept on the device, apply: the tables,
    lengths, refcounts and LIFO free list equal the reference's caches after each request
    rewinds its rejected suffix (or releases, once finished), in request order."""
    rng = np.random.default_rng(5)
    B, K1, ps, MP, cap = 300, 5, 16, 80, 300 * 80
    ctx = rng.integers(1, 1000, B)
    pool = oracle.PagePoolRef(ps)
    caches = [oracle.PagedCacheRef(pool) for _ in range(B)]
    dt = DevicePageTable(B, MP, ps, cap, device=cuda)
    for b in range(B):
        caches[b].append_chunk(int(ctx[b]))
    dt.append(torch.from_numpy(ctx.astype(np.int32)).to(cuda))
    for step in range(3):
        for b in range(B):
            if caches[b].offset:
                caches[b].append_chunk(K1)
        live = torch.tensor([K1 if c.offset else 0 for c in caches], dtype=torch.int32, device=cuda)
        dt.append(live)
        cand, ver = _random_batch(rng, B, K1, 6)
        active = np.array([1 if c.offset else 0 for c in caches], dtype=np.int32)
        res = verify_accept(torch.from_numpy(cand).to(cuda), torch.from_numpy(ver).to(cuda), eos_id=3,
                            active=torch.from_numpy(active).to(cuda))
        dt.apply_verify(res)
        dt.check_status()
        for b in range(B):
            if not active[b]:
                continue
            _, _, rw, _, fin = oracle.spec_accept_ref(cand[b].tolist(), ver[b].tolist(), 3)
            if fin:
                caches[b].release()
            else:
                caches[b].rewind(rw)
        for b in range(B):
            row = dt.block_table[b].tolist()
            assert row[:caches[b].num_pages] == caches[b].page_ids, (step, b)
            assert all(x == -1 for x in row[caches[b].num_pages:]), (step, b)
        assert dt.context_lens.tolist() == [c.offset for c in caches]
        assert dt.free_list() == pool.free_page_ids
        rc = dt.refcount.tolist()
        assert all(rc[p] == pool.ref_counts.get(p, 0) for p in range(pool.num_pages))
