"""Pins the oracle of the W4A16 quantized matmul (oracle_quantized_matmul, a C restatement
of QuantizedMatmul::eval_cpu, quantized_matmul.cpp:80-148).

The reference's tests (tests/test_quantized_matmul.py:6-47) compare its op with
mx.quantized_matmul on an identity input (exact: the output is the dequantised weight
matrix) and on a random normal input (atol 0.5); both are re-run here against a float64
closed form of the same affine 4-bit format.
"""

import numpy as np
import pytest

OR_F16, OR_BF16 = 1, 2


def _raw(x, code):
    from oracle import oracle as o

    return x.astype(np.float16) if code == OR_F16 else o.f32_to_bf16_bits(x.astype(np.float32))


def _f32(raw, code):
    from oracle import oracle as o

    return o.to_f32(raw, code)


def _dequant(packed, scales, biases):
    K, W = packed.shape
    q = np.zeros((K, W * 8), dtype=np.float64)
    for j in range(8):
        q[:, j::8] = (packed >> np.uint32(4 * j)) & np.uint32(15)
    s = np.repeat(scales.astype(np.float64), 128, axis=1)
    b = np.repeat(biases.astype(np.float64), 128, axis=1)
    return q * s + b


def _problem(rng, K, N, code):
    from oracle import oracle as o

    packed, s, b = o.quantize_w4_ref(rng.standard_normal((K, N)).astype(np.float32))
    s_raw, b_raw = _raw(s, code), _raw(b, code)
    return packed, s_raw, b_raw


@pytest.mark.parametrize("code", [OR_F16, OR_BF16], ids=["f16", "bf16"])
def test_identity_input_gives_dequantised_weights(oracle, code):
    """test_quantized_matmul.py:11-12,38-39: a = eye(128) -> out = dequantised weights^T."""
    rng = np.random.default_rng(code)
    K, N = 5, 128
    packed, s_raw, b_raw = _problem(rng, K, N, code)
    a = _raw(np.eye(N, dtype=np.float32), code)
    out = oracle.quantized_matmul_ref(a, code, packed, s_raw, b_raw)
    deq = _dequant(packed, _f32(s_raw, code), _f32(b_raw, code))  # exact q*s, one rounding for + b
    expect = _raw(deq.T.astype(np.float32), code)
    np.testing.assert_array_equal(out, expect)


@pytest.mark.parametrize("code", [OR_F16, OR_BF16], ids=["f16", "bf16"])
@pytest.mark.parametrize("shape", [(3, 128, 5), (4, 384, 17), (1, 2560, 32)])
def test_random_input_matches_closed_form(oracle, code, shape):
    """test_quantized_matmul.py:14-15,41-46 (random normal input), float64 reference."""
    M, N, K = shape
    rng = np.random.default_rng(M * N + K)
    packed, s_raw, b_raw = _problem(rng, K, N, code)
    a = _raw(rng.standard_normal((M, N)).astype(np.float32), code)
    out = _f32(oracle.quantized_matmul_ref(a, code, packed, s_raw, b_raw), code)
    ref = _f32(a, code).astype(np.float64) @ _dequant(packed, _f32(s_raw, code), _f32(b_raw, code)).T
    ulp = 2.0 ** -7 if code == OR_BF16 else 2.0 ** -10
    np.testing.assert_allclose(out, ref, rtol=ulp, atol=1e-4 * np.abs(ref).max() + 1e-6)


def test_packing_roundtrip(oracle):
    rng = np.random.default_rng(9)
    w = rng.standard_normal((7, 256)).astype(np.float32)
    packed, s, b = oracle.quantize_w4_ref(w)
    deq = _dequant(packed, s, b)
    assert packed.dtype == np.uint32 and packed.shape == (7, 32)
    assert np.abs(deq - w).max() <= np.repeat(s, 128, axis=1).max() / 2 + 1e-6
