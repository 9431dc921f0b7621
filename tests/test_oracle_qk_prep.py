"""Pins the oracle of the fused q/k norm + RoPE + paged write (oracle_qk_norm_rope_write).

The reference's own RoPE tests compare its custom RoPE with the closed-form rotation of
mx.fast.rope (tests/test_rope.py:8-50: B 1, 8 heads, head dim 4, tables of 20 rows,
10 tokens, base 10000, with and without an offset; tests/test_batching.py:48-54 with
one offset per request), at the tolerances of tests/utils.py:25-33.  They are re-run
here on the oracle against a float64 closed form.  RMSNorm is pinned the same way
(float64 mean of squares), the paged write against a numpy scatter and the int8
quantiser restatement, and the torch RoPE tables of the host package against the
oracle's tables.
"""

import numpy as np
import pytest

OR_F32, OR_F16, OR_BF16, OR_I8 = 0, 1, 2, 3
TOLS = {OR_F32: dict(rtol=1e-5, atol=5e-6), OR_F16: dict(rtol=5e-2, atol=1e-3)}


def _raw(x64, code):
    """float64 values -> raw oracle form of dtype code (bf16 as uint16 bits)."""
    from oracle import oracle as o

    if code == OR_F32:
        return x64.astype(np.float32)
    if code == OR_F16:
        return x64.astype(np.float16)
    return o.f32_to_bf16_bits(x64.astype(np.float32))


def _f64(raw, code):
    from oracle import oracle as o

    return o.to_f32(raw, code).astype(np.float64)


def _rope64(x, pos, dims, base, traditional):
    """Closed-form rotation (mx.fast.rope definition) in float64; x [T, H, D], pos [T]."""
    half = dims // 2
    theta = pos[:, None].astype(np.float64) * np.power(float(base), -np.arange(half) / half)[None, :]
    c, s = np.cos(theta)[:, None, :], np.sin(theta)[:, None, :]
    if traditional:
        x1, x2 = x[..., 0::2], x[..., 1::2]
        return np.stack([x1 * c - x2 * s, x1 * s + x2 * c], axis=-1).reshape(x.shape)
    x1, x2 = x[..., :half], x[..., half:]
    return np.concatenate([x1 * c - x2 * s, x1 * s + x2 * c], axis=-1)


def _run(oracle, q, k, v, code, pos, traditional, table_rows, base=10000, wq=None, wk=None, eps=1e-6,
         P=1, ps=4, kv_code=None, slots=None, scale_code=None):
    T, Hq, D = q.shape
    Hkv = k.shape[1]
    kv_code = code if kv_code is None else kv_code
    cos_t, sin_t = oracle.rope_tables_ref(D, table_rows, base)
    pool_dtype = {OR_F32: np.float32, OR_F16: np.float16, OR_BF16: np.uint16, OR_I8: np.int8}[kv_code]
    kp = np.zeros((P, Hkv, ps, D), dtype=pool_dtype)
    vp = np.zeros_like(kp)
    ks = vs = None
    scale_code = code if scale_code is None else scale_code
    if kv_code == OR_I8:
        sdt = {OR_F32: np.float32, OR_F16: np.float16, OR_BF16: np.uint16}[scale_code]
        ks = np.zeros((P, Hkv, ps, 1), dtype=sdt)
        vs = np.zeros_like(ks)
    if slots is None:
        slots = np.full(T, -1, dtype=np.int64)
    q_out, err = oracle.qk_norm_rope_write_ref(q, k, v, code, wq, wk, eps, cos_t, sin_t, traditional, pos, kp, vp,
                                               kv_code, ks, vs, scale_code, slots)
    return q_out, err, kp, vp, ks, vs


@pytest.mark.parametrize("code", [OR_F32, OR_F16], ids=["f32", "f16"])
@pytest.mark.parametrize("traditional", [False, True], ids=["default", "traditional"])
@pytest.mark.parametrize("with_offset", [True, False], ids=["with_offset", "without_offset"])
def test_rope_matches_closed_form(oracle, code, traditional, with_offset):
    """tests/test_rope.py:8-50 of the reference, re-run on the oracle (RoPE alone)."""
    rng = np.random.default_rng(1 + 2 * traditional + with_offset)
    H, D, MAX, L, BASE = 8, 4, 20, 10, 10000
    for _ in range(20):
        start = int(rng.integers(0, MAX - L)) if with_offset else 0
        pos = np.arange(start, start + L, dtype=np.int32)
        x = _raw(rng.uniform(size=(L, H, D)), code)
        q_out, err, *_ = _run(oracle, x, x[:, :1], x[:, :1], code, pos, traditional, MAX, BASE)
        assert err == 0
        ref = _rope64(_f64(x, code), pos, D, BASE, traditional)
        np.testing.assert_allclose(_f64(q_out, code), ref, **TOLS[code])


@pytest.mark.parametrize("traditional", [False, True], ids=["default", "traditional"])
def test_rope_multiple_offsets(oracle, traditional):
    """tests/test_batching.py:48-54: one offset per request in one call."""
    rng = np.random.default_rng(5)
    B, L, H, D, MAX = 3, 4, 8, 4, 40
    offsets = [0, 7, 29]
    pos = np.concatenate([np.arange(o, o + L) for o in offsets]).astype(np.int32)
    x = rng.uniform(size=(B * L, H, D)).astype(np.float32)
    q_out, err, *_ = _run(oracle, x, x[:, :1], x[:, :1], OR_F32, pos, traditional, MAX)
    assert err == 0
    np.testing.assert_allclose(q_out, _rope64(x.astype(np.float64), pos, D, 10000, traditional), **TOLS[OR_F32])


@pytest.mark.parametrize("code", [OR_F16, OR_BF16], ids=["f16", "bf16"])
@pytest.mark.parametrize("D", [64, 128, 4])
def test_rms_norm_matches_closed_form(oracle, code, D):
    """layers/layernorm.py:4-14: x * rsqrt(mean(x^2) + eps) * w, within one rounding of dtype
    (position 0 makes the rotation the identity)."""
    rng = np.random.default_rng(D)
    T, H, eps = 7, 5, 1e-6
    x = _raw(rng.standard_normal((T, H, D)) * rng.uniform(0.01, 20, size=(T, H, 1)), code)
    w = _raw(rng.uniform(0.5, 1.5, size=D), code)
    pos = np.zeros(T, dtype=np.int32)
    q_out, err, *_ = _run(oracle, x, x[:, :1], x[:, :1], code, pos, False, 4, wq=w, wk=w[:], eps=eps)
    assert err == 0
    x64 = _f64(x, code)
    ref = x64 / np.sqrt((x64 ** 2).mean(-1, keepdims=True) + eps) * _f64(w, code)
    ulp = 2.0 ** -7 if code == OR_BF16 else 2.0 ** -10
    np.testing.assert_allclose(_f64(q_out, code), ref, rtol=ulp, atol=1e-6)


def test_sum_order_is_the_lane_tree(oracle):
    """The oracle sums squares in the 32-lane tree order; on values whose squares sum
    exactly the order does not matter, so the result equals the plain formula."""
    D = 128
    x = np.full((1, 1, D), 2.0, dtype=np.float32)
    w = np.ones(D, dtype=np.float32)
    q_out, err, *_ = _run(oracle, x, x, x, OR_F32, np.zeros(1, np.int32), False, 4, wq=w, wk=w, eps=0.0)
    assert err == 0
    np.testing.assert_array_equal(q_out, np.ones_like(x))


@pytest.mark.parametrize("kv_code", [OR_BF16, OR_I8], ids=["bf16", "int8"])
def test_paged_write(oracle, kv_code):
    """Rotated K and raw V land at slot = page * page_size + offset; slot -1 is skipped;
    int8 pools hold _quantize_page_slice of the rounded rows."""
    rng = np.random.default_rng(11)
    T, Hq, Hkv, D, P, ps = 9, 4, 2, 64, 5, 4
    q = _raw(rng.standard_normal((T, Hq, D)), OR_BF16)
    k = _raw(rng.standard_normal((T, Hkv, D)) * 3, OR_BF16)
    v = _raw(rng.standard_normal((T, Hkv, D)), OR_BF16)
    w = _raw(rng.uniform(0.5, 1.5, size=D), OR_BF16)
    pos = rng.integers(0, 30, size=T).astype(np.int32)
    slots = rng.permutation(P * ps)[:T].astype(np.int64)
    slots[3] = -1
    q_out, err, kp, vp, ks, vs = _run(oracle, q, k, v, OR_BF16, pos, False, 32, wq=w, wk=w, P=P, ps=ps,
                                      kv_code=kv_code, slots=slots)
    assert err == 0
    # K rotated exactly as a q head with the k weights: run k through the q side
    k_rot, _, *_ = _run(oracle, k, k[:, :1], k[:, :1], OR_BF16, pos, False, 32, wq=w, wk=w)
    for t in range(T):
        s = int(slots[t])
        if s < 0:
            continue
        pid, off = s // ps, s % ps
        if kv_code == OR_I8:
            qk, sk = oracle.quantize_int8_ref(k_rot[t], OR_BF16)
            qv, sv = oracle.quantize_int8_ref(v[t], OR_BF16)
            np.testing.assert_array_equal(kp[pid, :, off], qk)
            np.testing.assert_array_equal(ks[pid, :, off], sk)
            np.testing.assert_array_equal(vp[pid, :, off], qv)
            np.testing.assert_array_equal(vs[pid, :, off], sv)
        else:
            np.testing.assert_array_equal(kp[pid, :, off], k_rot[t])
            np.testing.assert_array_equal(vp[pid, :, off], v[t])
    written = np.zeros((P, ps), dtype=bool)
    for s in slots[slots >= 0]:
        written[s // ps, s % ps] = True
    assert not kp.transpose(0, 2, 1, 3)[~written].any()


def test_out_of_range_position_and_page_flag(oracle):
    x = np.ones((2, 1, 4), dtype=np.float32)
    _, err, *_ = _run(oracle, x, x, x, OR_F32, np.array([0, 20], np.int32), False, 20)
    assert err == 1
    _, err, *_ = _run(oracle, x, x, x, OR_F32, np.array([0, 1], np.int32), False, 20, P=1, ps=4,
                      slots=np.array([1, 4], np.int64))
    assert err == 1


def test_torch_rope_tables_match_oracle_tables(oracle):
    """The host package's RoPE (rotary_embedding.py:28-44 restated in torch) and the
    oracle's numpy restatement both build fp32 tables within the fp32 rounding of the
    angle (pos * inv_freq, about rows * 2^-24 rad) of the float64 closed form; the
    libm pow / cos / sin of the two libraries may differ in the last place."""
    from nano_vllm_b200.layers.rotary_embedding import RoPE

    for dims, rows, base in [(128, 4096, 1000000), (64, 512, 10000), (4, 20, 10000)]:
        half = dims // 2
        theta = np.arange(rows)[:, None] * np.power(float(base), -np.arange(half) / half)[None, :]
        atol = max(2e-6, rows * 2.0 ** -22)
        rope = RoPE(dims, rows, base)
        c, s = oracle.rope_tables_ref(dims, rows, base)
        for table, ref in [(rope.cos_freqs.numpy(), np.cos(theta)), (c, np.cos(theta)),
                           (rope.sin_freqs.numpy(), np.sin(theta)), (s, np.sin(theta))]:
            assert table.dtype == np.float32 and table.shape == (rows, half)
            np.testing.assert_allclose(table, ref, rtol=0, atol=atol)
