"""The division-free int8 rounding of the kernels (nvm_common.cuh quantize_i8_fast),
restated in numpy fp32 (IEEE round to nearest even for +, -, *, / and the reciprocal):
t = fl(x * fl(1 / s)) is rounded through the 1.5 * 2^23 shifter and the integer read
from the sum's bits; wherever t lies at least 2^-14 from every half-integer this equals
rint(fl(x / s)), the reference's quotient (cache/paged.py:152-158), and elsewhere the
kernels divide.  Checked on random rows and on rows built a few ulps from half-integer
quotients."""

import numpy as np

MAGIC = np.float32(12582912.0)  # 1.5 * 2^23


def _check(x: np.ndarray, s: np.ndarray):
    r = np.float32(1.0) / s
    t = x * r
    f = t + MAGIC
    n = f - MAGIC
    fast = np.abs(t - n) < np.float32(0.5 - 2.0 ** -14)
    q = f.view(np.int32) - np.int32(0x4B400000)
    exact = np.rint(x / s)
    assert np.array_equal(q[fast].astype(np.float64), exact[fast].astype(np.float64))
    assert np.array_equal(n[fast], exact[fast])
    return fast.mean()


def test_guarded_product_rounds_like_quotient():
    rng = np.random.default_rng(0)
    rows, D = 20000, 128
    x = (rng.standard_normal((rows, D)) * rng.uniform(0.01, 50, (rows, 1))).astype(np.float32)
    amax = np.abs(x).max(axis=1, keepdims=True)
    s = (amax / np.float32(127)).astype(np.float32)
    assert _check(x, s) > 0.999


def test_guarded_product_near_half_integers():
    rng = np.random.default_rng(1)
    rows, D = 20000, 128
    A = rng.uniform(0.5, 100.0, (rows, 1)).astype(np.float32)
    s = (A / np.float32(127)).astype(np.float32)
    k = rng.integers(-126, 126, (rows, D)).astype(np.float64)
    x = ((k + 0.5) * s.astype(np.float64)).astype(np.float32)
    n = rng.integers(-4, 5, (rows, D))
    for step in range(4):
        x = np.where(n > step, np.nextafter(x, np.float32(np.inf)), x)
        x = np.where(n < -step, np.nextafter(x, np.float32(-np.inf)), x)
    x[:, 0] = A[:, 0]
    assert _check(x, s) < 0.5  # most of these take the division
