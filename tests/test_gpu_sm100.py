"""GPU parity of the tcgen05/TMEM prefill kernel (flash_sm100.cu) against the oracle.

Prefill-shaped calls (>= 64 query rows per head, 16-bit Q/K/V, head dim 128) take
this kernel: dense causal / full attention and chunked prefill over paged context.
"""

import pytest
import torch

from gpu_helpers import TOL16, assert_close, oracle_paged, random_paged_problem
from nano_vllm_b200 import flash_attention, paged_attention
from nano_vllm_b200 import _native as nv

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("dims", [(1, 4, 2, 256, 256), (2, 8, 2, 200, 333), (1, 2, 1, 128, 128), (1, 8, 8, 64, 512)])
@pytest.mark.parametrize("causal", [True, False])
def test_dense_prefill(cuda, oracle, dtype, dims, causal):
    B, Hq, Hkv, L, S = dims
    gen = torch.Generator().manual_seed(L * 7 + S)
    q = torch.randn(B, Hq, L, 128, generator=gen).to(dtype)
    k = torch.randn(B, Hkv, S, 128, generator=gen).to(dtype)
    v = torch.randn(B, Hkv, S, 128, generator=gen).to(dtype)
    mask = "causal" if causal else None
    out = flash_attention(q.cuda(), k.cuda(), v.cuda(), mask=mask, out_dtype=torch.float32)
    ref = oracle.flash_attention_ref(q.float().numpy(), k.float().numpy(), v.float().numpy(), mask=mask,
                                     nthreads=8)
    assert_close(out, ref, TOL16)
    assert nv.device_error(cuda) == 0


@pytest.mark.parametrize("holes", [False, True])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_paged_chunked_prefill(cuda, oracle, holes, dtype):
    gen = torch.Generator().manual_seed(31 + holes)
    prob = random_paged_problem(gen, 3, 8, 2, 192, 128, 16, dtype, 192, 900, holes=holes)
    out = paged_attention(prob["q"], prob["kp"], prob["vp"], prob["bt"], prob["cl"], 16, mask="causal")
    assert_close(out, oracle_paged(oracle, prob), TOL16)
    assert nv.device_error(cuda) == 0


def test_matches_mma_path(cuda, monkeypatch):
    gen = torch.Generator().manual_seed(5)
    prob = random_paged_problem(gen, 2, 16, 4, 384, 128, 16, torch.bfloat16, 600, 2000)
    args = (prob["q"], prob["kp"], prob["vp"], prob["bt"], prob["cl"], 16)
    a = paged_attention(*args, mask="causal")
    monkeypatch.setenv("NVM_ATTN_NO_SM100", "1")
    b = paged_attention(*args, mask="causal")
    torch.testing.assert_close(a, b, atol=2e-3, rtol=1e-2)


def test_repeated_calls_stable(cuda):
    gen = torch.Generator().manual_seed(9)
    q = torch.randn(2, 8, 512, 128, generator=gen).bfloat16().cuda()
    k = torch.randn(2, 2, 512, 128, generator=gen).bfloat16().cuda()
    v = torch.randn(2, 2, 512, 128, generator=gen).bfloat16().cuda()
    first = flash_attention(q, k, v, mask="causal")
    for _ in range(5):
        assert torch.equal(flash_attention(q, k, v, mask="causal"), first)
    assert nv.device_error(cuda) == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_paged_rows_without_keys(cuda, oracle, dtype):
    """Rows that see no key come out as zeros: context shorter than the chunk (causal
    limit below 0), an empty sequence, and rows whose visible keys are all holes."""
    gen = torch.Generator().manual_seed(77)
    B, Hq, Hkv, L, D, ps = 3, 8, 2, 192, 128, 16
    ctx = torch.tensor([100, 0, 300], dtype=torch.int32)
    pages = [(int(c) + ps - 1) // ps for c in ctx]
    MP = max(pages)
    P = sum(pages) + 2
    perm = torch.randperm(P, generator=gen)
    bt = torch.full((B, MP), -1, dtype=torch.int32)
    k = 0
    for b in range(B):
        bt[b, :pages[b]] = perm[k:k + pages[b]].to(torch.int32)
        k += pages[b]
    bt[2, :8] = -1  # keys 0..127 of sequence 2 missing: its rows 0..19 see only holes
    kp = torch.randn(P, Hkv, ps, D, generator=gen).to(dtype)
    vp = torch.randn(P, Hkv, ps, D, generator=gen).to(dtype)
    q = torch.randn(B, Hq, L, D, generator=gen).to(dtype)
    prob = dict(q=q.cuda(), kp=kp.cuda(), vp=vp.cuda(), ks=None, vs=None, bt=bt.cuda(), cl=ctx.cuda(), ps=ps)
    out = paged_attention(prob["q"], prob["kp"], prob["vp"], prob["bt"], prob["cl"], ps, mask="causal")
    ref = oracle_paged(oracle, prob)
    assert_close(out, ref, TOL16)
    got = out.cpu()
    assert torch.count_nonzero(got[0, :, :92]) == 0
    assert torch.count_nonzero(got[1]) == 0
    assert torch.count_nonzero(got[2, :, :20]) == 0
    assert nv.device_error(cuda) == 0


def test_dense_negative_scale(cuda, oracle):
    """A scale <= 0 is outside the tcgen05 kernel's contract (it takes row maxima
    before scaling); such calls take another kernel and still match."""
    gen = torch.Generator().manual_seed(3)
    q = torch.randn(1, 4, 256, 128, generator=gen).bfloat16()
    k = torch.randn(1, 2, 256, 128, generator=gen).bfloat16()
    v = torch.randn(1, 2, 256, 128, generator=gen).bfloat16()
    out = flash_attention(q.cuda(), k.cuda(), v.cuda(), scale=-0.05, mask="causal", out_dtype=torch.float32)
    ref = oracle.flash_attention_ref(q.float().numpy(), k.float().numpy(), v.float().numpy(), scale=-0.05,
                                     mask="causal", nthreads=8)
    assert_close(out, ref, TOL16)


@pytest.mark.parametrize("kind", ["dense", "chunked", "grouped"])
def test_pv_issue_order_bit_identical(cuda, monkeypatch, kind):
    """S_{j+2} issued right behind PV_j (NVM_SM100_PV_WAIT=0, relying on in-order
    execution of one thread's tcgen05.mma) gives the same bits as the default, which
    waits for PV_j to complete before S_{j+2} overwrites P_j."""
    gen = torch.Generator().manual_seed(17)
    if kind == "dense":
        q = torch.randn(2, 8, 1024, 128, generator=gen).bfloat16().cuda()
        k = torch.randn(2, 2, 1024, 128, generator=gen).bfloat16().cuda()
        v = torch.randn(2, 2, 1024, 128, generator=gen).bfloat16().cuda()
        run = lambda: flash_attention(q, k, v, mask="causal")  # noqa: E731
    else:
        L = 384 if kind == "chunked" else 5
        prob = random_paged_problem(gen, 4, 16, 4, L, 128, 16, torch.bfloat16, 600, 3000)
        run = lambda: paged_attention(prob["q"], prob["kp"], prob["vp"], prob["bt"], prob["cl"], 16,  # noqa: E731
                                      mask="causal")
    monkeypatch.setenv("NVM_SM100_PV_WAIT", "1")
    a = run()
    monkeypatch.setenv("NVM_SM100_PV_WAIT", "0")
    b = run()
    assert torch.equal(a, b)
    assert nv.device_error(cuda) == 0
