"""GPU parity of the two-query-tile tcgen05 kernel (flash_2q.cu) against the oracle.

With NVM_ATTN_2Q=1, prefill with at least 256 query rows per head (16-bit, head dim
128) takes this kernel: one CTA per (q head, 256-row block), 128-key K/V tiles shared by both query
tiles.  Dense causal / full attention (square and L < S, a partial last row block) and
chunked prefill over paged context (holes, an empty sequence); the order check runs the
MMA sequence with an explicit completion wait before each S overwrites P and must give
the same bits.
"""

import pytest
import torch

from gpu_helpers import TOL16, assert_close, oracle_paged, random_paged_problem
from nano_vllm_b200 import flash_attention, paged_attention
from nano_vllm_b200 import _native as nv

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _two_tile_kernel(monkeypatch):
    """The two-tile kernel is opt-in; every test here runs it."""
    monkeypatch.setenv("NVM_ATTN_2Q", "1")

DENSE = [(1, 4, 2, 256, 256), (2, 8, 2, 320, 320), (1, 4, 1, 300, 700), (1, 2, 1, 1024, 1024),
         (2, 4, 4, 512, 2048)]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("dims", DENSE, ids=lambda d: "x".join(map(str, d)))
@pytest.mark.parametrize("causal", [True, False])
def test_dense(cuda, oracle, dtype, dims, causal):
    B, Hq, Hkv, L, S = dims
    gen = torch.Generator().manual_seed(L * 3 + S + causal)
    q = torch.randn(B, Hq, L, 128, generator=gen).to(dtype)
    k = torch.randn(B, Hkv, S, 128, generator=gen).to(dtype)
    v = torch.randn(B, Hkv, S, 128, generator=gen).to(dtype)
    mask = "causal" if causal else None
    out = flash_attention(q.cuda(), k.cuda(), v.cuda(), mask=mask, out_dtype=torch.float32)
    ref = oracle.flash_attention_ref(q.float().numpy(), k.float().numpy(), v.float().numpy(), mask=mask,
                                     nthreads=8)
    assert_close(out, ref, TOL16)
    assert nv.device_error(cuda) == 0


@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float16])
def test_dense_16bit_out(cuda, oracle, out_dtype):
    gen = torch.Generator().manual_seed(2)
    q = torch.randn(1, 8, 512, 128, generator=gen).bfloat16()
    k = torch.randn(1, 2, 512, 128, generator=gen).bfloat16()
    v = torch.randn(1, 2, 512, 128, generator=gen).bfloat16()
    out = flash_attention(q.cuda(), k.cuda(), v.cuda(), mask="causal", out_dtype=out_dtype)
    ref = oracle.flash_attention_ref(q.float().numpy(), k.float().numpy(), v.float().numpy(), mask="causal",
                                     nthreads=8)
    assert_close(out, ref, TOL16)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("L,lo,hi", [(256, 256, 700), (300, 300, 1500), (512, 512, 2000)])
@pytest.mark.parametrize("holes", [False, True])
def test_paged_chunked(cuda, oracle, dtype, L, lo, hi, holes):
    gen = torch.Generator().manual_seed(L + hi + holes)
    prob = random_paged_problem(gen, 3, 8, 2, L, 128, 16, dtype, lo, hi, holes=holes, empty=True)
    out = paged_attention(prob["q"], prob["kp"], prob["vp"], prob["bt"], prob["cl"], 16, mask="causal")
    assert_close(out, oracle_paged(oracle, prob), TOL16)
    assert nv.device_error(cuda) == 0


def test_explicit_order_wait_same_bits(cuda, monkeypatch):
    gen = torch.Generator().manual_seed(8)
    q = torch.randn(2, 8, 1024, 128, generator=gen).bfloat16().cuda()
    k = torch.randn(2, 2, 1024, 128, generator=gen).bfloat16().cuda()
    v = torch.randn(2, 2, 1024, 128, generator=gen).bfloat16().cuda()
    a = flash_attention(q, k, v, mask="causal")
    monkeypatch.setenv("NVM_2Q_SAFE_ORDER", "1")
    b = flash_attention(q, k, v, mask="causal")
    assert torch.equal(a, b)
    for _ in range(3):
        monkeypatch.setenv("NVM_2Q_SAFE_ORDER", "0")
        assert torch.equal(a, flash_attention(q, k, v, mask="causal"))
    assert nv.device_error(cuda) == 0


def test_matches_one_tile_kernel(cuda, monkeypatch):
    gen = torch.Generator().manual_seed(4)
    prob = random_paged_problem(gen, 2, 16, 4, 384, 128, 16, torch.bfloat16, 600, 2000)
    args = (prob["q"], prob["kp"], prob["vp"], prob["bt"], prob["cl"], 16)
    a = paged_attention(*args, mask="causal")
    monkeypatch.setenv("NVM_ATTN_2Q", "0")
    b = paged_attention(*args, mask="causal")
    torch.testing.assert_close(a, b, atol=2e-3, rtol=1e-2)
