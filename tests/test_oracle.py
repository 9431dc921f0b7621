"""Pins the CPU oracle (oracle/nvm_oracle.c + oracle/oracle.py) before it is trusted.

The reference ships no golden vectors and cannot run here (MLX / Metal only), so the
oracle is pinned by re-running the reference's own tests on it, with numpy-seeded
data at the same shapes and tolerances:

* tests/test_paged_attention.py:105-137  paged vs dense flash attention (ps 4, 3+3 tokens)
* tests/test_paged_attention.py:140-188  batched decode with an empty slot
* tests/test_paged_kv_int8.py:7-46       int8 decode vs dequantised grouped SDPA
* tests/test_flash_attention.py:8-43,127-171  flash vs SDPA, modes no_mask/mask/causal
plus the committed fixtures of tests/golden/ (make_golden.py) and an independent
numpy restatement of the int8 quantiser.
"""

import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _chunk(rng, length, H=2, D=4, dtype=np.float32):
    k = rng.standard_normal((1, H, length, D)).astype(dtype)
    v = rng.standard_normal((1, H, length, D)).astype(dtype)
    return k, v


def test_paged_matches_dense_flash(oracle, rng):
    store = oracle.PagedStoreRef(page_size=4)
    cache = oracle.PagedCacheRef(store.pool)
    k1, v1 = _chunk(rng, 3)
    k2, v2 = _chunk(rng, 3)
    store.write(cache, k1, v1)
    store.write(cache, k2, v2)
    q = rng.standard_normal((1, 4, 3, 4)).astype(np.float32)
    dk, dv = store.gather_dense(cache)
    dense = oracle.flash_attention_ref(q, dk, dv, mask="causal")
    bt = np.array(cache.block_table(), dtype=np.int32)
    cl = np.array([cache.offset], dtype=np.int32)
    paged = oracle.paged_attention_ref(q, store.key_pages, store.value_pages, bt, cl, 4, mask="causal")
    assert bt.tolist() == [[0, 1]]
    assert cl.tolist() == [6]
    assert store.key_pages.shape == (2, 2, 4, 4)
    np.testing.assert_allclose(paged, dense, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(paged, oracle.grouped_sdpa_ref(q, dk, dv, mask="causal"), rtol=1e-5, atol=1e-6)


def test_batched_decode_with_empty_slot(oracle, rng):
    store = oracle.PagedStoreRef(page_size=4)
    first = oracle.PagedCacheRef(store.pool)
    second = oracle.PagedCacheRef(store.pool)
    store.write(first, *_chunk(rng, 3))
    store.write(second, *_chunk(rng, 6))
    store.write(first, *_chunk(rng, 1))
    store.write(second, *_chunk(rng, 1))
    caches = [first, None, second]
    max_pages = max(c.num_pages for c in caches if c is not None)
    bt = np.array([c.page_ids + [-1] * (max_pages - c.num_pages) if c else [-1] * max_pages for c in caches],
                  dtype=np.int32)
    cl = np.array([c.offset if c else 0 for c in caches], dtype=np.int32)
    q = rng.standard_normal((3, 4, 1, 4)).astype(np.float32)
    out = oracle.paged_attention_ref(q, store.key_pages, store.value_pages, bt, cl, 4, mask="causal")
    assert cl.tolist() == [4, 0, 7]
    assert bt.shape == (3, 2)
    assert bt.tolist()[1] == [-1, -1]
    assert store.key_pages.shape == (3, 2, 4, 4)
    for i in (0, 2):
        dk, dv = store.gather_dense(caches[i])
        ref = oracle.grouped_sdpa_ref(q[i:i + 1], dk, dv, mask="causal")
        np.testing.assert_allclose(out[i:i + 1], ref, rtol=1e-5, atol=1e-6)
    np.testing.assert_array_equal(out[1], 0.0)


def test_int8_decode_matches_dequantised_dense(oracle, rng):
    store = oracle.PagedStoreRef(page_size=4, kv_bits=8, is_bf16=True)
    cache = oracle.PagedCacheRef(store.pool)
    for _ in range(2):
        k = oracle.f32_to_bf16_bits(rng.standard_normal((1, 2, 3, 16)).astype(np.float32))
        v = oracle.f32_to_bf16_bits(rng.standard_normal((1, 2, 3, 16)).astype(np.float32))
        store.write(cache, k, v)
    q = rng.standard_normal((1, 4, 1, 16)).astype(np.float32)
    dk, dv = store.gather_dense(cache)
    dense = oracle.grouped_sdpa_ref(q, dk, dv, mask="causal")
    bt = np.array(cache.block_table(), dtype=np.int32)
    cl = np.array([cache.offset], dtype=np.int32)
    paged = oracle.paged_attention_ref(q, store.key_pages, store.value_pages, bt, cl, 4, store.key_scales,
                                       store.value_scales, mask="causal", scales_are_bf16=True)
    assert store.key_pages.dtype == np.int8 and store.value_pages.dtype == np.int8
    assert store.key_scales.shape == (2, 2, 4, 1)
    np.testing.assert_allclose(paged, dense, rtol=1e-4, atol=1e-4)


def test_int8_multi_token_dequantises_pool(oracle, rng):
    """attention.py:204-215: int8 with L > 1 equals fp32 paged attention on the dequantised pool."""
    store = oracle.PagedStoreRef(page_size=4, kv_bits=8)
    cache = oracle.PagedCacheRef(store.pool)
    store.write(cache, *_chunk(rng, 7, D=16, dtype=np.float16))
    q = rng.standard_normal((1, 4, 3, 16)).astype(np.float32)
    bt = np.array(cache.block_table(), dtype=np.int32)
    cl = np.array([cache.offset], dtype=np.int32)
    out = oracle.paged_attention_ref(q, store.key_pages, store.value_pages, bt, cl, 4, store.key_scales,
                                     store.value_scales, mask="causal")
    dk, dv = store.gather_dense(cache)
    np.testing.assert_allclose(out, oracle.grouped_sdpa_ref(q, dk, dv, mask="causal"), rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("shape", [(6, 3, 2, 5, 3, 1), (18, 6, 7, 5, 3, 10), (28, 4, 16, 128, 16, 3),
                                   (1, 1, 5, 7, 4, 1)])
@pytest.mark.parametrize("mode", ["no_mask", "mask", "causal"])
def test_flash_matches_sdpa(oracle, rng, shape, mode):
    Hq, H, L, E, S, B = shape
    if mode == "causal" and L > S:
        pytest.skip("the reference runs causal only with L <= S")
    for _ in range(5):
        q = rng.uniform(size=(B, Hq, L, E)).astype(np.float32)
        k = rng.uniform(size=(B, H, S, E)).astype(np.float32)
        v = rng.uniform(size=(B, H, S, E)).astype(np.float32)
        mask = {"no_mask": None, "causal": "causal",
                "mask": rng.uniform(size=(B, Hq, L, S)).astype(np.float32)}[mode]
        out = oracle.flash_attention_ref(q, k, v, scale=0.9, mask=mask)
        ref = oracle.grouped_sdpa_ref(q, k, v, scale=0.9, mask=mask)
        np.testing.assert_allclose(out, ref, rtol=5e-2, atol=1e-3)
        np.testing.assert_allclose(out, ref, rtol=1e-5, atol=1e-5)


def test_paged_edge_cases(oracle, rng):
    """Holes (-1) are skipped, ctx <= 0 gives zeros, ctx beyond capacity is clipped."""
    P, H, ps, D = 6, 2, 4, 8
    kp = rng.standard_normal((P, H, ps, D)).astype(np.float32)
    vp = rng.standard_normal((P, H, ps, D)).astype(np.float32)
    q = rng.standard_normal((3, 4, 1, D)).astype(np.float32)
    bt = np.array([[2, -1, 4], [0, 1, 3], [5, -1, -1]], dtype=np.int32)
    cl = np.array([12, 0, 40], dtype=np.int32)
    out = oracle.paged_attention_ref(q, kp, vp, bt, cl, ps)
    np.testing.assert_array_equal(out[1], 0.0)
    keys0 = np.concatenate([kp[2], kp[4]], axis=1)[None]  # hole skipped
    vals0 = np.concatenate([vp[2], vp[4]], axis=1)[None]
    np.testing.assert_allclose(out[0:1], oracle.grouped_sdpa_ref(q[0:1], keys0, vals0), rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(out[2:3], oracle.grouped_sdpa_ref(q[2:3], kp[5][None], vp[5][None]), rtol=1e-5,
                               atol=1e-6)


@pytest.mark.parametrize("code", [0, 1, 2])
def test_quantizer_matches_numpy_restatement(oracle, rng, code):
    x = (rng.standard_normal((64, 128)) * rng.uniform(0.01, 20, size=(64, 1))).astype(np.float32)
    x[3] = 0.0  # amax == 0 -> scale 1
    x[5, :4] = [2.5 * 127 / 127, -0.5, 0.5, 1.5]  # exercise ties after scaling
    if code == 1:
        raw = x.astype(np.float16)
        xf = raw.astype(np.float32)
    elif code == 2:
        raw = oracle.f32_to_bf16_bits(x)
        xf = oracle.bf16_bits_to_f32(raw)
    else:
        raw = x
        xf = x
    q, s = oracle.quantize_int8_ref(raw, code)
    amax = np.abs(xf).max(axis=-1, keepdims=True)
    s_ref = np.where(amax > 0, amax / np.float32(127.0), np.float32(1.0)).astype(np.float32)
    q_ref = np.clip(np.round(xf / s_ref), -127, 127).astype(np.int8)
    np.testing.assert_array_equal(q, q_ref)
    if code == 0:
        np.testing.assert_array_equal(s, s_ref)
    elif code == 1:
        np.testing.assert_array_equal(s, s_ref.astype(np.float16))
    else:
        np.testing.assert_array_equal(s, oracle.f32_to_bf16_bits(s_ref))
    assert np.abs(q.astype(np.int32)).max() <= 127


def test_round_half_even_ties(oracle):
    # x / s lands exactly on .5: numpy/MLX round-half-to-even -> 0, 2, -2, 2.
    x = np.array([[0.5, 1.5, -2.5, 2.5, 127.0]], dtype=np.float32)  # amax 127 -> s = 1
    q, s = oracle.quantize_int8_ref(x, 0)
    assert s.ravel().tolist() == [1.0]
    assert q.ravel().tolist() == [0, 2, -2, 2, 127]


def test_golden_fixtures(oracle):
    files = sorted(f for f in os.listdir(GOLDEN) if f.endswith(".npz"))
    assert files, "tests/golden has no fixtures; run tests/golden/make_golden.py"
    import sys

    sys.path.insert(0, GOLDEN)
    import make_golden

    for f in files:
        data = dict(np.load(os.path.join(GOLDEN, f)))
        got = make_golden.run_case(oracle, data)
        for key, val in got.items():
            np.testing.assert_array_equal(val, data[key], err_msg=f"{f}:{key}")
