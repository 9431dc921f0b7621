"""GPU parity of the W4A16 quantized matmul (nvm_w4a16_matmul) with the oracle restatement
of QuantizedMatmul::eval_cpu.

The kernel contracts each 128-element group on the tensor cores and applies scale and
bias once per group (s * sum(a q) + b * sum(a)); the oracle dequantises every element and
sums in order.  Both accumulate in fp32, so results agree to fp32 rounding before the
final rounding to bf16 / fp16: the bar is one unit in the last place of the output dtype
(plus 1e-4 of the output range for cancellation).  The identity input of the reference's
test (test_quantized_matmul.py:11-12) is bit-exact.
"""

import numpy as np
import pytest
import torch

from gpu_helpers import to_np
from nano_vllm_b200.layers.linear import QuantizedWeights, quantized_linear, quantized_matmul

pytestmark = pytest.mark.gpu

CODE = {torch.float16: 1, torch.bfloat16: 2}


def _to_torch(raw, dtype, cuda):
    if dtype == torch.bfloat16:
        return torch.from_numpy(np.ascontiguousarray(raw).view(np.int16)).view(torch.bfloat16).to(cuda)
    return torch.from_numpy(np.ascontiguousarray(raw)).to(cuda)


def _problem(oracle, rng, M, N, K, dtype, cuda, identity=False):
    code = CODE[dtype]
    packed, s, b = oracle.quantize_w4_ref(rng.standard_normal((K, N)).astype(np.float32))
    conv = (lambda x: x.astype(np.float16)) if code == 1 else (lambda x: oracle.f32_to_bf16_bits(x))
    s_raw, b_raw = conv(s), conv(b)
    a = np.eye(N, dtype=np.float32)[:M] if identity else rng.standard_normal((M, N)).astype(np.float32)
    a_raw = conv(a)
    ref = oracle.quantized_matmul_ref(a_raw, code, packed, s_raw, b_raw, nthreads=oracle.max_threads())
    t = dict(a=_to_torch(a_raw, dtype, cuda), b=torch.from_numpy(packed.view(np.int32)).to(cuda),
             s=_to_torch(s_raw, dtype, cuda), bi=_to_torch(b_raw, dtype, cuda))
    return t, ref


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "f16"])
def test_identity_bit_exact(cuda, oracle, dtype):
    rng = np.random.default_rng(1)
    t, ref = _problem(oracle, rng, 128, 128, 5, dtype, cuda, identity=True)
    out = quantized_matmul(t["s"], t["bi"], 128, 4, t["a"], t["b"], transpose_b=True)
    np.testing.assert_array_equal(to_np(out), ref)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "f16"])
@pytest.mark.parametrize("M,N,K", [(1, 128, 5), (3, 256, 17), (8, 2560, 40), (9, 384, 16), (16, 1024, 33),
                                   (33, 512, 24), (1, 9728, 64)])
def test_random_matches_oracle(cuda, oracle, dtype, M, N, K):
    rng = np.random.default_rng(M * 7 + N + K)
    t, ref = _problem(oracle, rng, M, N, K, dtype, cuda)
    out = quantized_matmul(t["s"], t["bi"], 128, 4, t["a"], t["b"], transpose_b=True)
    got = oracle.to_f32(to_np(out), CODE[dtype]).astype(np.float64)
    r = oracle.to_f32(ref, CODE[dtype]).astype(np.float64)
    ulp = 2.0 ** -7 if dtype == torch.bfloat16 else 2.0 ** -10
    np.testing.assert_allclose(got, r, rtol=ulp, atol=1e-4 * np.abs(r).max() + 1e-6)


def test_batched_leading_dims_and_linear(cuda, oracle):
    """[B, 1, N] decode activations (quantized_linear reshapes to [-1, N]) plus a bias."""
    rng = np.random.default_rng(5)
    t, ref = _problem(oracle, rng, 6, 512, 20, torch.bfloat16, cuda)
    w = QuantizedWeights(t["s"], t["bi"], 128, 4, t["b"])
    bias = torch.randn(20, device=cuda).bfloat16()
    out = quantized_linear(t["a"].reshape(6, 1, 512), w, bias)
    assert out.shape == (6, 1, 20)
    base = quantized_matmul(t["s"], t["bi"], 128, 4, t["a"], t["b"], True)
    assert torch.equal(out.reshape(6, 20), base + bias)


def test_argument_errors(cuda):
    a = torch.zeros(2, 128, dtype=torch.bfloat16, device=cuda)
    b = torch.zeros(4, 16, dtype=torch.int32, device=cuda)
    s = torch.ones(4, 1, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(RuntimeError, match="bits must be 4"):
        quantized_matmul(s, s, 128, 8, a, b, True)
    with pytest.raises(RuntimeError, match="group_size must be 128"):
        quantized_matmul(s, s, 64, 4, a, b, True)
    with pytest.raises(RuntimeError, match="must be transposed"):
        quantized_matmul(s, s, 128, 4, a, b, False)
    with pytest.raises(RuntimeError, match="same dtype as scales"):
        quantized_matmul(s, s, 128, 4, a.half(), b, True)


@pytest.mark.parametrize("split", [1, 2, 3, 8])
def test_cluster_split_matches_oracle(cuda, oracle, monkeypatch, split):
    """The groups of each 16-row tile split over a thread-block cluster of `split` CTAs
    (forced here; by default only projections with few tiles split) give the oracle's
    result to the same tolerance, including ragged rows and a group count that does not
    divide evenly."""
    monkeypatch.setenv("NVM_W4_SPLIT", str(split))
    rng = np.random.default_rng(split)
    for M, N, K in [(3, 4096, 40), (12, 2560, 17)]:
        t, ref = _problem(oracle, rng, M, N, K, torch.bfloat16, cuda)
        out = quantized_matmul(t["s"], t["bi"], 128, 4, t["a"], t["b"], transpose_b=True)
        got = oracle.to_f32(to_np(out), 2).astype(np.float64)
        r = oracle.to_f32(ref, 2).astype(np.float64)
        np.testing.assert_allclose(got, r, rtol=2.0 ** -7, atol=1e-4 * np.abs(r).max() + 1e-6)
