"""GPU parity of the paged KV scatter-write and int8 quantise-on-write (bit-exact)."""

import numpy as np
import pytest
import torch

from gpu_helpers import to_np
from nano_vllm_b200 import BatchingKvCache, TinyKvPagedCache, TinyKvPagedPool, write_slots

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("D", [4, 64, 128, 100])
def test_copy_scatter_bit_exact(cuda, dtype, D):
    gen = torch.Generator().manual_seed(D)
    P, H, ps, T = 9, 3, 16, 40
    kp = torch.randn(P, H, ps, D, generator=gen).to(dtype).cuda()
    vp = torch.randn(P, H, ps, D, generator=gen).to(dtype).cuda()
    k = torch.randn(T, H, D, generator=gen).to(dtype).cuda()
    v = torch.randn(T, H, D, generator=gen).to(dtype).cuda()
    slots = torch.randperm(P * ps, generator=gen)[:T]
    slots[::7] = -1  # skipped tokens
    ref_k, ref_v = kp.clone(), vp.clone()
    for t in range(T):
        s = int(slots[t])
        if s >= 0:
            ref_k[s // ps, :, s % ps] = k[t]
            ref_v[s // ps, :, s % ps] = v[t]
    write_slots(k, v, slots.cuda(), kp, vp)
    assert torch.equal(kp, ref_k) and torch.equal(vp, ref_v)


def test_strided_source(cuda):
    """[1, H, S, D] chunks are read through their strides (no copy)."""
    gen = torch.Generator().manual_seed(0)
    kp = torch.zeros(4, 2, 8, 64, dtype=torch.bfloat16, device="cuda")
    vp = torch.zeros_like(kp)
    k = torch.randn(1, 2, 11, 64, generator=gen).to(torch.bfloat16).cuda()
    v = torch.randn(1, 2, 11, 64, generator=gen).to(torch.bfloat16).cuda()
    slots = torch.arange(11, device="cuda") + 3
    write_slots(k[0].transpose(0, 1), v[0].transpose(0, 1), slots, kp, vp)
    flat_k = kp.permute(0, 2, 1, 3).reshape(32, 2, 64)
    assert torch.equal(flat_k[3:14], k[0].transpose(0, 1))


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_int8_quantise_bit_exact(cuda, oracle, dtype):
    gen = torch.Generator().manual_seed(7)
    P, H, ps, D, T = 6, 2, 16, 128, 50
    x = (torch.randn(T, H, D, generator=gen) * torch.rand(T, H, 1, generator=gen) * 30).to(dtype)
    x[5] = 0  # all-zero rows -> scale 1, values 0
    xv = (torch.randn(T, H, D, generator=gen) * 4).to(dtype)
    kp = torch.zeros(P, H, ps, D, dtype=torch.int8, device="cuda")
    vp = torch.zeros_like(kp)
    ks = torch.ones(P, H, ps, 1, dtype=dtype, device="cuda")
    vs = torch.ones_like(ks)
    slots = torch.randperm(P * ps, generator=gen)[:T]
    write_slots(x.cuda(), xv.cuda(), slots.cuda(), kp, vp, ks, vs)
    code = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}[dtype]
    for src, pages, scales in ((x, kp, ks), (xv, vp, vs)):
        q_ref, s_ref = oracle.quantize_int8_ref(to_np(src), code)
        pg, sc = to_np(pages), to_np(scales)
        for t in range(T):
            s = int(slots[t])
            np.testing.assert_array_equal(pg[s // ps, :, s % ps], q_ref[t])
            np.testing.assert_array_equal(sc[s // ps, :, s % ps], s_ref[t])


def _tie_rows(dtype, gen):
    """[8, 2, 128] rows whose x / s are exact half-integers: the amax element is
    254/256 (so s = amax / 127 = 1/128 exactly) and the others are (2k + 1) / 256 with
    random signs, i.e. x / s = k + 1/2.  In fp32, tokens 1 and 2 move every non-amax
    element one ulp up / down (quotients just off the tie)."""
    vals = torch.tensor([254.0 / 256] + [(2 * k + 1) / 256 for k in range(127)], dtype=torch.float64)
    rows = []
    for t in range(8):
        sign = torch.where(torch.rand(2, 128, generator=gen) < 0.5, -1.0, 1.0).double()
        x = vals.repeat(2, 1) * sign
        if dtype == torch.float32 and t in (1, 2):
            step = torch.full_like(x[:, 1:], float("inf") if t == 1 else 0.0).float()
            x32 = x.float()
            x32[:, 1:] = torch.nextafter(x32[:, 1:], torch.where(x32[:, 1:] > 0, step, -step))
            x = x32.double()
        rows.append(x)
    return torch.stack(rows).to(dtype)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_int8_rounding_ties_bit_exact(cuda, oracle, dtype):
    """Half-integer quotients (and one ulp either side of them): the division-free
    rounding of the kernels must agree with round-half-even of the IEEE x / s."""
    gen = torch.Generator().manual_seed(11)
    x = _tie_rows(dtype, gen)
    T, H, D, P, ps = 8, 2, 128, 2, 16
    kp = torch.zeros(P, H, ps, D, dtype=torch.int8, device="cuda")
    vp = torch.zeros_like(kp)
    ks = torch.ones(P, H, ps, 1, dtype=dtype, device="cuda")
    vs = torch.ones_like(ks)
    slots = torch.arange(T, dtype=torch.int64) * 3
    write_slots(x.cuda(), x.flip(0).cuda(), slots.cuda(), kp, vp, ks, vs)
    code = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}[dtype]
    for src, pages, scales in ((x, kp, ks), (x.flip(0), vp, vs)):
        q_ref, s_ref = oracle.quantize_int8_ref(to_np(src), code)
        pg, sc = to_np(pages), to_np(scales)
        for t in range(T):
            s = int(slots[t])
            np.testing.assert_array_equal(pg[s // ps, :, s % ps], q_ref[t])
            np.testing.assert_array_equal(sc[s // ps, :, s % ps], s_ref[t])


def _near_tie_rows(gen, T, H, D):
    """fp32 rows with random non-power-of-two scales whose quotients x / s sit within a
    few ulps of half-integers: amax A in [0.5, 100) as element 0, the others
    fl((k + 1/2) * fl(A / 127)) moved by -4..4 ulps, k in [-126, 125]."""
    A = (torch.rand(T, H, 1, generator=gen, dtype=torch.float64) * 99.5 + 0.5).float()
    s = (A.double() / 127).float().double()
    k = torch.randint(-126, 126, (T, H, D), generator=gen).double()
    x = ((k + 0.5) * s).float()
    n = torch.randint(-4, 5, (T, H, D), generator=gen)
    for step in range(4):
        up = n > step
        down = n < -step
        x = torch.where(up, torch.nextafter(x, torch.full_like(x, float("inf"))), x)
        x = torch.where(down, torch.nextafter(x, torch.full_like(x, -float("inf"))), x)
    x[:, :, 0] = A[:, :, 0] * torch.where(torch.rand(T, H, generator=gen) < 0.5, -1.0, 1.0)
    return x


def test_int8_near_ties_random_scales_bit_exact(cuda, oracle):
    """Quotients a few ulps from half-integers under arbitrary scales: the product with
    the reciprocal scale must round like the IEEE quotient (the kernels fall back to the
    division near a half-integer)."""
    gen = torch.Generator().manual_seed(23)
    T, H, D, P, ps = 64, 4, 128, 8, 16
    x = _near_tie_rows(gen, T, H, D)
    xv = _near_tie_rows(gen, T, H, D)
    kp = torch.zeros(P, H, ps, D, dtype=torch.int8, device="cuda")
    vp = torch.zeros_like(kp)
    ks = torch.ones(P, H, ps, 1, dtype=torch.float32, device="cuda")
    vs = torch.ones_like(ks)
    slots = torch.randperm(P * ps, generator=gen)[:T]
    write_slots(x.cuda(), xv.cuda(), slots.cuda(), kp, vp, ks, vs)
    for src, pages, scales in ((x, kp, ks), (xv, vp, vs)):
        q_ref, s_ref = oracle.quantize_int8_ref(to_np(src), 0)
        pg, sc = to_np(pages), to_np(scales)
        for t in range(T):
            sl = int(slots[t])
            np.testing.assert_array_equal(pg[sl // ps, :, sl % ps], q_ref[t])
            np.testing.assert_array_equal(sc[sl // ps, :, sl % ps], s_ref[t])


def test_paged_cache_matches_full_cache(cuda):
    gen = torch.Generator().manual_seed(3)
    pool = TinyKvPagedPool(page_size=4)
    paged = TinyKvPagedCache(pool)
    fk = fv = None  # the dense history: every chunk concatenated along the sequence
    total = 0
    for n in [3, 2, 5]:
        k = torch.randn(1, 2, n, 4, generator=gen).cuda()
        v = torch.randn(1, 2, n, 4, generator=gen).cuda()
        fk = k if fk is None else torch.cat([fk, k], dim=2)
        fv = v if fv is None else torch.cat([fv, v], dim=2)
        pk, pv, plen, _ = paged.update_and_fetch(k, v)
        total += n
        assert plen == total
        assert paged.num_pages == (total + 3) // 4
        assert [pool.read_page(p)[0].shape[2] for p in paged.page_ids] == [4] * paged.num_pages
        assert torch.equal(pk, fk) and torch.equal(pv, fv)


def test_int8_pool_matches_oracle_store(cuda, oracle):
    """Pages, scales and pool shapes of a kv_bits=8 pool equal the oracle's restatement."""
    gen = torch.Generator().manual_seed(4)
    pool = TinyKvPagedPool(page_size=4, kv_bits=8)
    cache = TinyKvPagedCache(pool)
    store = oracle.PagedStoreRef(page_size=4, kv_bits=8, is_bf16=True)
    rcache = oracle.PagedCacheRef(store.pool)
    for n in [3, 3, 7, 1]:
        k = torch.randn(1, 2, n, 16, generator=gen).to(torch.bfloat16)
        v = torch.randn(1, 2, n, 16, generator=gen).to(torch.bfloat16)
        cache.update_and_fetch_paged(k.cuda(), v.cuda())
        store.write(rcache, to_np(k), to_np(v))
    assert cache.page_ids == rcache.page_ids
    np.testing.assert_array_equal(to_np(pool.key_pages), store.key_pages)
    np.testing.assert_array_equal(to_np(pool.value_pages), store.value_pages)
    np.testing.assert_array_equal(to_np(pool.key_scales), store.key_scales)
    np.testing.assert_array_equal(to_np(pool.value_scales), store.value_scales)


def test_batching_cache_single_write(cuda, oracle):
    """update_and_fetch_paged: same ids/lengths as per-request appends, one kernel write."""
    gen = torch.Generator().manual_seed(5)
    pool = TinyKvPagedPool(page_size=4, reserve_pages=64)
    reqs = [TinyKvPagedCache(pool) for _ in range(3)]
    for r, n in zip(reqs, [5, 2, 9]):
        r.update_and_fetch(*(torch.randn(1, 2, n, 8, generator=gen).cuda() for _ in range(2)))
    batch = BatchingKvCache(max_active_requests=4, max_seq_len=8)
    for i, r in enumerate(reqs):
        batch.add_request(r, [0, 1, 3][i])
    k = torch.randn(4, 2, 3, 8, generator=gen).cuda()
    v = torch.randn(4, 2, 3, 8, generator=gen).cuda()
    meta = batch.update_and_fetch_paged(k, v, mask="causal")
    assert meta.context_lens.tolist() == [8, 5, 0, 12]
    for slot, r in zip([0, 1, 3], reqs):
        dk, dv = r.gather_dense()
        assert torch.equal(dk[0, :, -3:], k[slot]) and torch.equal(dv[0, :, -3:], v[slot])
        row = meta.block_table[slot].tolist()
        assert row[:r.num_pages] == r.page_ids and all(x == -1 for x in row[r.num_pages:])
    assert meta.block_table[2].tolist() == [-1] * meta.block_table.shape[1]
