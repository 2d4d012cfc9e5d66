"""CPU check of the exact-product argument the window refit kernels rely on
(no GPU needed).

The window stores record keys, record corrections and compensators as
binary16.  A product of two binary16 values has at most 11 + 11 = 22
significant bits and a magnitude between 2^-48 and 65504^2, inside fp32's
normal range, so the fp32 product is exact: RN(a * b) = a * b.  The
reference's RN(x + RN(a * b)) is then fma(a, b, x) for every fp32 x, and the
refit's record update RN(RN(d S) + RN(k c)) takes one rounded product and one
fma (csrc/window.cuh: window_dense_kernel, window_fold_kernel).

This test multiplies every finite binary16 value (both zeros and the
subnormals included) by a stratified set of partners covering the whole
binary16 range and its extremes, in fp32, and compares with the exact fp64
product: value and sign.
"""

from __future__ import annotations

import numpy as np


def finite_halves() -> np.ndarray:
    h = np.arange(1 << 16, dtype=np.uint32).astype(np.uint16).view(np.float16)
    return h[np.isfinite(h)].astype(np.float32)


def test_every_finite_binary16_value_is_covered():
    a = finite_halves()
    assert a.size == 2 * (31 * 1024)  # 31 finite exponents x 1024 significands, both signs
    assert np.float32(65504.0) in a and np.float32(2.0 ** -24) in a


def test_binary16_products_are_exact_in_fp32():
    a = finite_halves()
    extremes = np.array([0.0, -0.0, 2.0 ** -24, -(2.0 ** -24), 1023 * 2.0 ** -24, 2.0 ** -14,
                         2047 * 2.0 ** -24, 1.0, 2047 / 1024, 65504.0, -65504.0,
                         2047 * 2.0 ** -10 * 2.0 ** 14], dtype=np.float32)
    b = np.unique(np.concatenate([a[::29], extremes]))
    assert np.all(np.isfinite(b.astype(np.float16)))  # every partner is a binary16 value
    b64 = b.astype(np.float64)
    for chunk in np.array_split(a, 64):
        p32 = chunk[:, None] * b[None, :]                      # fp32, round to nearest
        p64 = chunk.astype(np.float64)[:, None] * b64[None, :]  # exact: 22 <= 53 bits
        assert np.array_equal(p32.astype(np.float64), p64)
        assert np.array_equal(np.signbit(p32), np.signbit(p64))
