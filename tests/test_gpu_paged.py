"""GPU parity of paged attention (libnvm_attn) against the oracle.

Covers the reference's own paged tests (restated on the product API), the committed
golden fixtures, a randomized sweep over dtypes / head dims / page sizes / query
lengths / causal modes with holes, empty rows and clipped contexts, the split-K
combine, and the BASELINE config shapes at reduced batch.  Tolerances: fp32 pages
1e-5 / 1e-6 (reference tests/utils.py), fp16/bf16/int8 max-abs 2e-3 + rel 1e-2.
"""

import os
import sys

import numpy as np
import pytest
import torch

from gpu_helpers import TOL16, TOL32, assert_close, oracle_paged, random_paged_problem, to_np
from nano_vllm_b200 import (BatchingKvCache, TinyKvPagedCache, TinyKvPagedPool, flash_attention, paged_attention,
                            scaled_dot_product_attention_grouped)
from nano_vllm_b200 import _native as nv

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _chunk(gen, n, H=2, D=4, dtype=torch.float32):
    return (torch.randn(1, H, n, D, generator=gen).to(dtype).cuda(),
            torch.randn(1, H, n, D, generator=gen).to(dtype).cuda())


def test_paged_matches_dense_flash(cuda):
    gen = torch.Generator().manual_seed(0)
    pool = TinyKvPagedPool(page_size=4)
    cache = TinyKvPagedCache(pool)
    cache.update_and_fetch(*_chunk(gen, 3))
    meta = cache.update_and_fetch_paged(*_chunk(gen, 3), mask="causal")
    q = torch.randn(1, 4, 3, 4, generator=gen).cuda()
    dk, dv = cache.gather_dense()
    dense = flash_attention(q, dk, dv, mask="causal")
    paged = paged_attention(q, meta.key_pages, meta.value_pages, meta.block_table, meta.context_lens,
                            meta.page_size, mask=meta.mask)
    assert meta.block_table.tolist() == [[0, 1]]
    assert meta.context_lens.tolist() == [6]
    assert tuple(meta.key_pages.shape) == (2, 2, 4, 4)
    torch.testing.assert_close(paged, dense, **TOL32)


def test_batched_paged_decode_with_empty_slot(cuda):
    gen = torch.Generator().manual_seed(1)
    pool = TinyKvPagedPool(page_size=4)
    first, second = TinyKvPagedCache(pool), TinyKvPagedCache(pool)
    first.update_and_fetch(*_chunk(gen, 3))
    second.update_and_fetch(*_chunk(gen, 6))
    batch = BatchingKvCache(max_active_requests=3, max_seq_len=16)
    batch.add_request(first, 0)
    batch.add_request(second, 2)
    keys = torch.zeros(3, 2, 1, 4, device="cuda")
    values = torch.zeros(3, 2, 1, 4, device="cuda")
    keys[0:1], values[0:1] = _chunk(gen, 1)
    keys[2:3], values[2:3] = _chunk(gen, 1)
    meta = batch.update_and_fetch_paged(keys, values, mask_length=1, mask="causal")
    q = torch.randn(3, 4, 1, 4, generator=gen).cuda()
    out = paged_attention(q, meta.key_pages, meta.value_pages, meta.block_table, meta.context_lens,
                          meta.page_size, mask=meta.mask)
    fk, fv = first.gather_dense()
    sk, sv = second.gather_dense()
    assert meta.context_lens.tolist() == [4, 0, 7]
    assert tuple(meta.block_table.shape) == (3, 2)
    assert meta.block_table.tolist()[1] == [-1, -1]
    assert tuple(meta.key_pages.shape) == (3, 2, 4, 4)
    torch.testing.assert_close(out[0:1], scaled_dot_product_attention_grouped(q[0:1], fk, fv, mask="causal"),
                               **TOL32)
    torch.testing.assert_close(out[2:3], scaled_dot_product_attention_grouped(q[2:3], sk, sv, mask="causal"),
                               **TOL32)
    assert (out[1] == 0).all()


def test_int8_decode_matches_dequantised_dense(cuda, oracle):
    gen = torch.Generator().manual_seed(2)
    pool = TinyKvPagedPool(page_size=4, kv_bits=8)
    cache = TinyKvPagedCache(pool)
    cache.update_and_fetch(*_chunk(gen, 3, D=16, dtype=torch.bfloat16))
    meta = cache.update_and_fetch_paged(*_chunk(gen, 3, D=16, dtype=torch.bfloat16), mask="causal")
    q = torch.randn(1, 4, 1, 16, generator=gen).cuda()
    dk, dv = cache.gather_dense()
    dense = scaled_dot_product_attention_grouped(q, dk, dv, mask="causal")
    out = paged_attention(q, meta.key_pages, meta.value_pages, meta.block_table, meta.context_lens,
                          meta.page_size, key_scales=meta.key_scales, value_scales=meta.value_scales,
                          mask=meta.mask)
    assert meta.key_pages.dtype == torch.int8 and meta.value_pages.dtype == torch.int8
    assert tuple(meta.key_scales.shape) == (2, 2, 4, 1)
    torch.testing.assert_close(out, dense, atol=1e-4, rtol=1e-4)


@pytest.mark.parametrize("name", ["paged_f16_decode", "paged_bf16_verify", "paged_i8_decode", "paged_i8_multi"])
def test_golden_paged(cuda, name):
    d = dict(np.load(os.path.join(GOLDEN, name + ".npz")))
    q = torch.from_numpy(d["q"]).cuda()
    if d["k"].dtype == np.uint16:
        kp = torch.from_numpy(d["k"].view(np.int16)).view(torch.bfloat16).cuda()
        vp = torch.from_numpy(d["v"].view(np.int16)).view(torch.bfloat16).cuda()
    else:
        kp, vp = torch.from_numpy(d["k"]).cuda(), torch.from_numpy(d["v"]).cuda()
    ks = torch.from_numpy(d["ks"]).cuda() if "ks" in d else None
    vs = torch.from_numpy(d["vs"]).cuda() if "vs" in d else None
    bt, cl = torch.from_numpy(d["bt"]).cuda(), torch.from_numpy(d["cl"]).cuda()
    out = paged_attention(q, kp, vp, bt, cl, kp.shape[2], ks, vs, mask="causal" if int(d["causal"]) else None)
    assert_close(out, d["out"], TOL16, name)


SWEEP = [
    # kv dtype, D, ps, Hq, Hkv, L, causal
    (torch.float32, 4, 4, 4, 2, 1, True),
    (torch.float32, 32, 8, 4, 2, 3, True),
    (torch.float16, 16, 4, 4, 2, 1, True),
    (torch.float16, 128, 16, 16, 8, 1, True),
    (torch.bfloat16, 128, 16, 32, 8, 1, True),
    (torch.bfloat16, 64, 16, 8, 1, 1, False),
    (torch.bfloat16, 128, 32, 32, 4, 5, True),
    (torch.float16, 128, 16, 12, 4, 4, True),
    (torch.bfloat16, 128, 16, 16, 2, 3, False),
    (torch.float16, 64, 64, 8, 2, 7, True),
    (torch.bfloat16, 96, 16, 4, 2, 2, True),  # D=96 -> generic kernel
    (torch.int8, 128, 16, 64, 8, 1, True),
    (torch.int8, 128, 16, 16, 4, 5, True),
    (torch.int8, 128, 32, 8, 8, 1, True),
    (torch.int8, 32, 4, 4, 2, 2, True),      # generic int8 path
    # multi-token rows on the n8 tile (at most eight query rows per kv head, causal
    # limits differing per row)
    (torch.bfloat16, 128, 16, 8, 4, 3, True),
    (torch.float16, 128, 16, 8, 2, 2, True),
    (torch.int8, 128, 16, 8, 4, 3, True),
    (torch.bfloat16, 64, 16, 4, 4, 5, True),
    (torch.float16, 128, 32, 6, 2, 2, False),
]


@pytest.mark.parametrize("case", SWEEP, ids=lambda c: f"{str(c[0]).split('.')[-1]}-D{c[1]}-ps{c[2]}-g{c[3]//c[4]}-L{c[5]}-{'c' if c[6] else 'nc'}")
def test_random_sweep(cuda, oracle, case):
    kvd, D, ps, Hq, Hkv, L, causal = case
    gen = torch.Generator().manual_seed(hash(case) % (2 ** 31))
    prob = random_paged_problem(gen, 5, Hq, Hkv, L, D, ps, kvd, 1, 300, holes=True, empty=True)
    mask = "causal" if causal else None
    out = paged_attention(prob["q"], prob["kp"], prob["vp"], prob["bt"], prob["cl"], ps, prob["ks"], prob["vs"],
                          mask=mask)
    ref = oracle_paged(oracle, prob, mask=mask)
    assert_close(out, ref, TOL32 if kvd == torch.float32 else TOL16)
    assert nv.device_error(cuda) == 0


@pytest.mark.parametrize("kvd", [torch.bfloat16, torch.int8])
def test_split_k_combine(cuda, oracle, kvd, monkeypatch):
    """Long contexts split into 16-tile chunks across CTAs; last-CTA merge; ticket reset."""
    monkeypatch.setenv("NVM_ATTN_CHUNK_TILES", "16")
    gen = torch.Generator().manual_seed(3)
    prob = random_paged_problem(gen, 6, 16, 4 if kvd == torch.int8 else 8, 1, 128, 16, kvd, 200, 2000, holes=True)
    for _ in range(3):  # tickets must be back at zero for the next call
        out = paged_attention(prob["q"], prob["kp"], prob["vp"], prob["bt"], prob["cl"], 16, prob["ks"],
                              prob["vs"], mask="causal")
        assert_close(out, oracle_paged(oracle, prob), TOL16)
    assert nv.device_error(cuda) == 0


@pytest.mark.parametrize("kvd", [torch.float16, torch.bfloat16, torch.int8])
@pytest.mark.parametrize("chunk_tiles", ["8", "16", "32"])
def test_cluster_merge_equals_workspace_merge(cuda, oracle, kvd, chunk_tiles, monkeypatch):
    """n8 decode split into 2..8 chunks: merged inside a thread-block cluster over
    distributed shared memory, or through the workspace -- the same operations in the
    same order, so bit-identical -- and both equal the oracle.  Ragged contexts (chunks
    without keys still join the cluster), holes, an empty sequence."""
    monkeypatch.setenv("NVM_ATTN_CHUNK_TILES", chunk_tiles)
    gen = torch.Generator().manual_seed(int(chunk_tiles) + 7)
    prob = random_paged_problem(gen, 9, 16, 8, 1, 128, 16, kvd, 1, 1024, holes=True, empty=True)
    args = (prob["q"], prob["kp"], prob["vp"], prob["bt"], prob["cl"], 16, prob["ks"], prob["vs"])
    outs = {}
    for mode in ("0", "2"):
        monkeypatch.setenv("NVM_ATTN_CLUSTER", mode)
        outs[mode] = [paged_attention(*args, mask="causal") for _ in range(2)]
    assert torch.equal(outs["0"][0], outs["2"][0]) and torch.equal(outs["2"][0], outs["2"][1])
    assert_close(outs["2"][0], oracle_paged(oracle, prob), TOL16)
    assert nv.device_error(cuda) == 0


def test_workspace_shared_across_shapes(cuda, oracle):
    """One cached workspace serves split-K calls of different shapes back to back."""
    gen = torch.Generator().manual_seed(21)
    probs = [random_paged_problem(gen, 16, 16, 8, 1, 128, 16, torch.float16, 128, 1024, spare_pages=64),
             random_paged_problem(gen, 40, 32, 8, 1, 128, 16, torch.bfloat16, 1000, 3000),
             random_paged_problem(gen, 3, 64, 8, 1, 128, 16, torch.int8, 2000, 5000)]
    for prob in probs + probs[::-1]:
        out = paged_attention(prob["q"], prob["kp"], prob["vp"], prob["bt"], prob["cl"], 16, prob["ks"], prob["vs"],
                              mask="causal")
        assert_close(out, oracle_paged(oracle, prob), TOL16)
    assert nv.device_error(cuda) == 0


def test_context_clipped_to_block_table(cuda, oracle):
    gen = torch.Generator().manual_seed(4)
    prob = random_paged_problem(gen, 3, 8, 2, 1, 128, 16, torch.float16, 40, 100)
    prob["cl"] = prob["cl"] + 1000  # longer than max_pages * page_size: clipped, causal offset uses ctx
    out = paged_attention(prob["q"], prob["kp"], prob["vp"], prob["bt"], prob["cl"], 16, mask="causal")
    assert_close(out, oracle_paged(oracle, prob), TOL16)


@pytest.mark.parametrize("out_dtype", [torch.float16, torch.bfloat16])
def test_out_dtype(cuda, oracle, out_dtype):
    gen = torch.Generator().manual_seed(5)
    prob = random_paged_problem(gen, 4, 16, 8, 1, 128, 16, torch.bfloat16, 30, 500)
    out = paged_attention(prob["q"], prob["kp"], prob["vp"], prob["bt"], prob["cl"], 16, mask="causal",
                          out_dtype=out_dtype)
    assert out.dtype == out_dtype
    assert_close(out, oracle_paged(oracle, prob), dict(atol=5e-3, rtol=1e-2))


def test_fp32_query_on_16bit_pages(cuda, oracle):
    """The reference passes fp32 queries; the kernel converts them to the page dtype."""
    gen = torch.Generator().manual_seed(6)
    prob = random_paged_problem(gen, 4, 16, 8, 1, 128, 16, torch.float16, 30, 500, q_dtype=torch.float32)
    out = paged_attention(prob["q"], prob["kp"], prob["vp"], prob["bt"], prob["cl"], 16, mask="causal")
    assert_close(out, oracle_paged(oracle, prob), TOL16)


# ---- BASELINE config shapes (reduced batch where the oracle would be slow) -----

@pytest.mark.parametrize("cfg", ["c1_decode_f16", "c3_decode_bf16", "c4_int8", "c5_verify", "c2b_chunked"])
def test_config_shapes(cuda, oracle, cfg):
    gen = torch.Generator().manual_seed(11)
    if cfg == "c1_decode_f16":
        prob = random_paged_problem(gen, 16, 16, 8, 1, 128, 16, torch.float16, 128, 1024, spare_pages=64)
    elif cfg == "c3_decode_bf16":
        prob = random_paged_problem(gen, 3, 32, 8, 1, 128, 16, torch.bfloat16, 4096, 12000)
    elif cfg == "c4_int8":
        prob = random_paged_problem(gen, 2, 64, 8, 1, 128, 16, torch.int8, 8192, 12000)
    elif cfg == "c5_verify":
        prob = random_paged_problem(gen, 6, 32, 4, 5, 128, 16, torch.bfloat16, 256, 4000)
    else:
        prob = random_paged_problem(gen, 1, 16, 4, 256, 128, 16, torch.bfloat16, 256 + 512, 256 + 1024)
    out = paged_attention(prob["q"], prob["kp"], prob["vp"], prob["bt"], prob["cl"], 16, prob["ks"], prob["vs"],
                          mask="causal")
    assert_close(out, oracle_paged(oracle, prob), TOL16, cfg)


def test_page_permutation_invariance(cuda):
    """Moving pages to other physical ids (and rewriting the block table) changes nothing."""
    gen = torch.Generator().manual_seed(12)
    prob = random_paged_problem(gen, 8, 32, 8, 1, 128, 16, torch.bfloat16, 500, 3000)
    out1 = paged_attention(prob["q"], prob["kp"], prob["vp"], prob["bt"], prob["cl"], 16, mask="causal")
    P = prob["kp"].shape[0]
    perm = torch.randperm(P, generator=gen).cuda()
    inv = torch.empty_like(perm)
    inv[perm] = torch.arange(P, device="cuda")
    kp2, vp2 = prob["kp"][perm], prob["vp"][perm]  # new id j holds old page perm[j]
    bt2 = torch.where(prob["bt"] >= 0, inv[prob["bt"].clamp(min=0).long()].to(torch.int32), prob["bt"])
    out2 = paged_attention(prob["q"], kp2, vp2, bt2, prob["cl"], 16, mask="causal")
    torch.testing.assert_close(out1, out2, atol=0, rtol=0)


def test_linearity_in_values(cuda):
    """Attention is linear in V for fixed scores: att(a*V1 + b*V2) = a*att(V1) + b*att(V2)."""
    gen = torch.Generator().manual_seed(13)
    prob = random_paged_problem(gen, 8, 32, 8, 1, 128, 16, torch.float16, 500, 3000)
    v2 = torch.randn(prob["vp"].shape, generator=gen).to(torch.float16).cuda()
    args = lambda v: (prob["q"], prob["kp"], v, prob["bt"], prob["cl"], 16)  # noqa: E731
    o1 = paged_attention(*args(prob["vp"]), mask="causal")
    o2 = paged_attention(*args(v2), mask="causal")
    o3 = paged_attention(*args((0.5 * prob["vp"].float() + 0.25 * v2.float()).half()), mask="causal")
    torch.testing.assert_close(o3, 0.5 * o1 + 0.25 * o2, atol=2e-3, rtol=1e-2)


def test_validation_errors(cuda):
    q = torch.zeros(1, 3, 1, 128, device="cuda")
    kp = torch.zeros(2, 2, 16, 128, device="cuda", dtype=torch.bfloat16)
    bt = torch.zeros(1, 2, dtype=torch.int32, device="cuda")
    cl = torch.ones(1, dtype=torch.int32, device="cuda")
    with pytest.raises(AssertionError):
        paged_attention(q, kp, kp, bt, cl, 16)
    with pytest.raises(RuntimeError, match="same dtype"):
        paged_attention(q[:, :2], kp, kp.float(), bt, cl, 16)


@pytest.mark.parametrize("variant", ["2", "7", "3", "4", "5"], ids=["ring2", "ring4", "ring6", "ring8", "w4ring4"])
@pytest.mark.parametrize("kvd", [torch.bfloat16, torch.int8])
def test_n8_ring_depths_match_oracle(cuda, oracle, kvd, variant, monkeypatch):
    """The n8 decode tile (no producer warp: each warp refills the ring stages it
    consumes) at every 2-warp ring depth that NVM_ATTN_DECODE_CFG can select and with 4
    warps of one stage each, on
    ragged split-K contexts with page holes and a row count that leaves the tile part empty."""
    monkeypatch.setenv("NVM_ATTN_DECODE_CFG", variant)
    monkeypatch.setenv("NVM_ATTN_CHUNK_TILES", "16")
    gen = torch.Generator().manual_seed(40 + int(variant))
    Hq, Hkv = (24, 4) if kvd == torch.int8 else (12, 4)  # 6 / 3 query rows per kv head
    prob = random_paged_problem(gen, 7, Hq, Hkv, 1, 128, 16, kvd, 1, 1500, holes=True, empty=True)
    for _ in range(2):
        out = paged_attention(prob["q"], prob["kp"], prob["vp"], prob["bt"], prob["cl"], 16, prob["ks"],
                              prob["vs"], mask="causal")
        assert_close(out, oracle_paged(oracle, prob), TOL16)
    assert nv.device_error(cuda) == 0
