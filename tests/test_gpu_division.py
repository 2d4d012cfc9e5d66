"""The quantizer's exact division (the two-term reciprocal of c and one fma
correction, used for every smoothed value s = R / c) against IEEE float32
division, on the device, over random and adversarial operands inside the
routine's documented range."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from gdn_state_codec import _native

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def device_quotients(a: np.ndarray, c: np.ndarray) -> np.ndarray:
    ta = torch.from_numpy(a).to(DEV)
    tc = torch.from_numpy(c).to(DEV)
    out = torch.empty_like(ta)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    status = _native.call("statecentric_gdn_state_codec_division_selftest_v1", stream,
                          ctypes.c_void_p(ta.data_ptr()), ctypes.c_void_p(tc.data_ptr()),
                          ctypes.c_void_p(out.data_ptr()), a.size)
    assert status == 0
    torch.cuda.synchronize()
    return out.cpu().numpy()


def random_floats(rng, n, lo_exp, hi_exp, all_ones_fraction=0.0):
    mant = rng.integers(0, 1 << 23, n, dtype=np.uint32)
    if all_ones_fraction:
        mask = rng.random(n) < all_ones_fraction
        mant[mask] = (1 << 23) - 1 - rng.integers(0, 4, mask.sum(), dtype=np.uint32)
    exp = rng.integers(lo_exp + 127, hi_exp + 127 + 1, n, dtype=np.uint32)
    sign = rng.integers(0, 2, n, dtype=np.uint32) << 31
    return (sign | (exp << 23) | mant).view(np.float32)


def check(a, c):
    with np.errstate(all="ignore"):
        want = (a / c).astype(np.float32)
    ok = np.isfinite(want) & (np.abs(want) >= np.float32(2.0 ** -125)) & (
        np.abs(a) >= np.float32(2.0 ** -102))
    got = device_quotients(a[ok].copy(), c[ok].copy())
    mism = int((got.view(np.uint32) != want[ok].view(np.uint32)).sum())
    assert mism == 0, f"{mism} of {ok.sum()} quotients differ from IEEE division"
    return int(ok.sum())


def test_random_wide_range():
    rng = np.random.default_rng(0)
    n = 1 << 24
    a = random_floats(rng, n, -90, 100)
    c = np.abs(random_floats(rng, n, -14, 100, all_ones_fraction=0.1))
    assert check(a, c) > n // 2


def test_codec_like_operands():
    """Smoothing in [1e-4, 1e3] and states in the benchmark distribution."""
    rng = np.random.default_rng(1)
    n = 1 << 24
    c = np.sqrt(10.0 ** rng.uniform(-8, 6, n)).astype(np.float32)
    a = (rng.standard_normal(n) * 10.0 ** (-3 * rng.random(n))).astype(np.float32)
    assert check(a, c) > n * 0.99


def test_quotients_near_rounding_midpoints():
    """a = RN(m * c) for m a float midpoint: quotients within a few ulp of a
    rounding boundary, where a faithful-only routine would fail."""
    rng = np.random.default_rng(2)
    n = 1 << 23
    q = np.abs(random_floats(rng, n, -20, 20))
    c = np.abs(random_floats(rng, n, -10, 10, all_ones_fraction=0.25))
    mid = q.astype(np.float64) * (1.0 + 2.0 ** -24)  # halfway to the next float
    a = (mid * c.astype(np.float64)).astype(np.float32)
    assert check(a, c) > n * 0.99
