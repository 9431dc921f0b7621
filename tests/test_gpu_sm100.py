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
