"""GPU parity of dense flash attention (prefill) against the oracle."""

import os

import numpy as np
import pytest
import torch

from gpu_helpers import TOL16, TOL32, assert_close
from nano_vllm_b200 import flash_attention, scaled_dot_product_attention_grouped

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.mark.parametrize("shape", [(6, 3, 2, 5, 3, 1), (18, 6, 7, 5, 3, 10), (28, 4, 16, 128, 16, 3),
                                   (1, 1, 5, 7, 4, 1)])
@pytest.mark.parametrize("mode", ["no_mask", "mask", "causal"])
def test_reference_flash_shapes(cuda, oracle, shape, mode):
    """tests/test_flash_attention.py:8-43 of the reference, fp32, scale 0.9."""
    Hq, H, L, E, S, B = shape
    if mode == "causal" and L > S:
        pytest.skip("the reference runs causal only with L <= S")
    gen = torch.Generator().manual_seed(sum(shape))
    for _ in range(10):
        q = torch.rand(B, Hq, L, E, generator=gen)
        k = torch.rand(B, H, S, E, generator=gen)
        v = torch.rand(B, H, S, E, generator=gen)
        mask = {"no_mask": None, "causal": "causal", "mask": torch.rand(B, Hq, L, S, generator=gen)}[mode]
        out = flash_attention(q.cuda(), k.cuda(), v.cuda(), scale=0.9,
                              mask=mask.cuda() if isinstance(mask, torch.Tensor) else mask)
        ref = oracle.flash_attention_ref(q.numpy(), k.numpy(), v.numpy(), scale=0.9,
                                         mask=mask.numpy() if isinstance(mask, torch.Tensor) else mask)
        assert_close(out, ref, TOL32)


@pytest.mark.parametrize("name", ["flash_mask", "flash_causal"])
def test_golden_flash(cuda, name):
    d = dict(np.load(os.path.join(GOLDEN, name + ".npz")))
    mask = "causal" if int(d["causal"]) else torch.from_numpy(d["mask"]).cuda()
    out = flash_attention(torch.from_numpy(d["q"]).cuda(), torch.from_numpy(d["k"]).cuda(),
                          torch.from_numpy(d["v"]).cuda(), scale=float(d["scale"]), mask=mask)
    assert_close(out, d["out"], TOL32)


def test_broadcast_mask_not_materialised(cuda, oracle):
    """A [L, S] mask broadcast over batch and heads is read through stride-0 views."""
    gen = torch.Generator().manual_seed(1)
    q = torch.randn(2, 4, 9, 32, generator=gen)
    k = torch.randn(2, 2, 13, 32, generator=gen)
    v = torch.randn(2, 2, 13, 32, generator=gen)
    m = torch.randn(9, 13, generator=gen)
    out = flash_attention(q.cuda(), k.cuda(), v.cuda(), mask=m.cuda())
    ref = oracle.flash_attention_ref(q.numpy(), k.numpy(), v.numpy(), mask=m.numpy())
    assert_close(out, ref, TOL32)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("dims", [(2, 8, 2, 256, 256), (1, 32, 8, 300, 300), (2, 4, 4, 64, 200), (1, 8, 2, 1, 77)])
@pytest.mark.parametrize("causal", [True, False])
def test_16bit_prefill(cuda, oracle, dtype, dims, causal):
    B, Hq, Hkv, L, S = dims
    gen = torch.Generator().manual_seed(B * 1000 + L)
    q = torch.randn(B, Hq, L, 128, generator=gen).to(dtype)
    k = torch.randn(B, Hkv, S, 128, generator=gen).to(dtype)
    v = torch.randn(B, Hkv, S, 128, generator=gen).to(dtype)
    mask = "causal" if causal else None
    out = flash_attention(q.cuda(), k.cuda(), v.cuda(), mask=mask, out_dtype=torch.float32)
    ref = oracle.flash_attention_ref(q.float().numpy(), k.float().numpy(), v.float().numpy(), mask=mask,
                                     nthreads=8)
    assert_close(out, ref, TOL16)


def test_grouped_sdpa_reference_helper(cuda):
    gen = torch.Generator().manual_seed(2)
    q = torch.randn(1, 4, 5, 16, generator=gen)
    k = torch.randn(1, 2, 7, 16, generator=gen)
    v = torch.randn(1, 2, 7, 16, generator=gen)
    out = flash_attention(q.cuda(), k.cuda(), v.cuda(), mask="causal")
    ref = scaled_dot_product_attention_grouped(q, k, v, mask="causal")
    torch.testing.assert_close(out.cpu(), ref, **TOL32)
