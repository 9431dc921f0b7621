"""GPU parity of the tcgen05 kernel's grouped mode (flash_sm100.cu) against the oracle.

Calls with 2..63 query tokens per sequence and at least 16 query rows per kv head
(g * L) run one tile per kv head holding its whole query group, split over keys into
chunks whose partial results the last chunk merges.  Reference semantics: causal key
limit l + ctx - L per query position l, holes skipped, rows that see no key are zeros.
"""

import pytest
import torch

from gpu_helpers import TOL16, assert_close, oracle_paged, random_paged_problem
from nano_vllm_b200 import flash_attention, paged_attention
from nano_vllm_b200 import _native as nv

pytestmark = pytest.mark.gpu


def _run(prob, **kw):
    return paged_attention(prob["q"], prob["kp"], prob["vp"], prob["bt"], prob["cl"], prob["ps"], mask="causal", **kw)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [(3, 32, 4, 5), (2, 16, 2, 2), (2, 8, 1, 8), (2, 8, 2, 33), (1, 32, 2, 10)])
@pytest.mark.parametrize("holes", [False, True])
def test_grouped_decode(cuda, oracle, dtype, shape, holes):
    B, Hq, Hkv, L = shape
    gen = torch.Generator().manual_seed(B * 1000 + Hq * 10 + L + holes)
    prob = random_paged_problem(gen, B, Hq, Hkv, L, 128, 16, dtype, L, 700, holes=holes)
    out = _run(prob)
    assert_close(out, oracle_paged(oracle, prob), TOL16)
    assert nv.device_error(cuda) == 0


@pytest.mark.parametrize("chunk_tiles", ["1", "2", "3"])
def test_grouped_split_k(cuda, oracle, monkeypatch, chunk_tiles):
    """Small forced chunks: many partials per kv head merged by the last chunk; a
    second identical call checks that the tickets were left at zero."""
    monkeypatch.setenv("NVM_SM100_CHUNK_TILES", chunk_tiles)
    gen = torch.Generator().manual_seed(int(chunk_tiles))
    prob = random_paged_problem(gen, 4, 16, 2, 5, 128, 16, torch.bfloat16, 5, 1500, holes=True, empty=True)
    first = _run(prob)
    assert_close(first, oracle_paged(oracle, prob), TOL16)
    second = _run(prob)
    assert torch.equal(first, second)
    assert nv.device_error(cuda) == 0


def test_grouped_rows_without_keys(cuda, oracle):
    gen = torch.Generator().manual_seed(4)
    B, Hq, Hkv, L, D, ps = 3, 16, 2, 8, 128, 16
    ctx = torch.tensor([3, 0, 200], dtype=torch.int32)  # 3 < L: positions 0..4 see nothing
    pages = [max((int(c) + ps - 1) // ps, 1) for c in ctx]
    MP, P = max(pages), sum(pages) + 1
    perm = torch.randperm(P, generator=gen)
    bt = torch.full((B, MP), -1, dtype=torch.int32)
    k = 0
    for b in range(B):
        bt[b, :pages[b]] = perm[k:k + pages[b]].to(torch.int32)
        k += pages[b]
    bt[2, :12] = -1  # keys 0..191 of sequence 2 missing: its positions 0..7 see only holes
    kp = torch.randn(P, Hkv, ps, D, generator=gen).bfloat16()
    vp = torch.randn(P, Hkv, ps, D, generator=gen).bfloat16()
    q = torch.randn(B, Hq, L, D, generator=gen).bfloat16()
    prob = dict(q=q.cuda(), kp=kp.cuda(), vp=vp.cuda(), ks=None, vs=None, bt=bt.cuda(), cl=ctx.cuda(), ps=ps)
    out = _run(prob)
    assert_close(out, oracle_paged(oracle, prob), TOL16)
    got = out.cpu()
    assert torch.count_nonzero(got[0, :, :5]) == 0
    assert torch.count_nonzero(got[1]) == 0
    assert nv.device_error(cuda) == 0


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
def test_grouped_two_row_tiles(cuda, oracle, out_dtype):
    """g * L = 160 rows: two tiles per kv head, the second holding 32 rows."""
    gen = torch.Generator().manual_seed(11)
    prob = random_paged_problem(gen, 2, 16, 1, 10, 128, 16, torch.bfloat16, 10, 900)
    out = _run(prob, out_dtype=out_dtype)
    assert out.dtype == out_dtype
    assert_close(out.float(), oracle_paged(oracle, prob), TOL16)
    assert nv.device_error(cuda) == 0


def test_grouped_dense_flash(cuda, oracle):
    gen = torch.Generator().manual_seed(21)
    q = torch.randn(2, 16, 6, 128, generator=gen).bfloat16()
    k = torch.randn(2, 2, 300, 128, generator=gen).bfloat16()
    v = torch.randn(2, 2, 300, 128, generator=gen).bfloat16()
    out = flash_attention(q.cuda(), k.cuda(), v.cuda(), mask="causal", out_dtype=torch.float32)
    ref = oracle.flash_attention_ref(q.float().numpy(), k.float().numpy(), v.float().numpy(), mask="causal",
                                     nthreads=8)
    assert_close(out, ref, TOL16)


def test_grouped_matches_mma_path(cuda, monkeypatch):
    gen = torch.Generator().manual_seed(6)
    prob = random_paged_problem(gen, 4, 32, 4, 5, 128, 16, torch.bfloat16, 200, 3000)
    a = _run(prob)
    monkeypatch.setenv("NVM_SM100_GROUPED", "0")
    b = _run(prob)
    torch.testing.assert_close(a, b, atol=2e-3, rtol=1e-2)


def test_grouped_dense_many_units(cuda, oracle):
    """Dense few-token calls with more units than the persistent grid (two CTAs per SM):
    CTAs walk the units by index and store rows directly."""
    gen = torch.Generator().manual_seed(31)
    q = torch.randn(200, 16, 4, 128, generator=gen).bfloat16()
    k = torch.randn(200, 2, 96, 128, generator=gen).bfloat16()
    v = torch.randn(200, 2, 96, 128, generator=gen).bfloat16()
    out = flash_attention(q.cuda(), k.cuda(), v.cuda(), mask="causal", out_dtype=torch.float32)
    ref = oracle.flash_attention_ref(q.float().numpy(), k.float().numpy(), v.float().numpy(), mask="causal",
                                     nthreads=8)
    assert_close(out, ref, TOL16)
    assert nv.device_error(cuda) == 0


def test_grouped_fp16_and_out_dtypes(cuda, oracle):
    gen = torch.Generator().manual_seed(41)
    prob = random_paged_problem(gen, 3, 16, 2, 4, 128, 16, torch.float16, 4, 1200, holes=True)
    for od in (torch.float32, torch.float16):
        out = _run(prob, out_dtype=od)
        assert out.dtype == od
        assert_close(out.float(), oracle_paged(oracle, prob), TOL16)
    assert nv.device_error(cuda) == 0
