"""CPU tests of the oracle (oracle/gdn_codec_oracle.c) against the reference.

The oracle is the checker of every GPU parity test, so it is pinned first:
  * against golden vectors produced by the reference library itself
    (tests/golden/make_golden.py: FromDenseBoundary -> Serialize, DenseState,
    ApplyToken of vLLM-HUST/gdn-state-codec native/src), and
  * when the reference library has been compiled here (oracle/_ref), against
    fresh calls into it on seeded heads, edge cases included.
The reference's own three test programs are run too when they were built.
"""

from __future__ import annotations

import subprocess

import numpy as np
import pytest

import oracle


def bits(a: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def assert_same_bits(name: str, got: np.ndarray, want: np.ndarray) -> None:
    got = np.asarray(got)
    want = np.asarray(want)
    assert got.shape == want.shape, f"{name}: shape {got.shape} != {want.shape}"
    if got.dtype == np.float32:
        diff = int((bits(got) != bits(want)).sum())
    else:
        diff = int((got != want).sum())
    assert diff == 0, f"{name}: {diff} of {got.size} elements differ"


def residuals(heads: dict) -> np.ndarray:
    n = heads["dense"].shape[0]
    return np.stack([oracle.rebuild_residual(heads["dense"][i], heads["compensator_keys"][i],
                                             heads["compensator_values"][i]) for i in range(n)])


def test_oracle_quantize_matches_reference_boundary(golden):
    """Quantizing the residual left by the reference's rank-4 fit reproduces
    the serialized boundary (capsule.cpp:140-225) bit for bit."""
    g = golden["heads"]
    z, c, b = oracle.quantize(residuals(g), "capsule")
    assert_same_bits("codes", z, g["codes"])
    assert_same_bits("smoothing", c, g["smoothing"])
    assert_same_bits("scales", b, g["scales"])


def test_oracle_dequantize_matches_dense_state(golden):
    """DenseState() of the reference (capsule.cpp:229-251, 337-352)."""
    g = golden["heads"]
    got = oracle.dequantize(g["codes"], g["smoothing"], g["scales"],
                            g["compensator_keys"], g["compensator_values"])
    assert_same_bits("DenseState", got, g["dense_state"])


def test_oracle_projection_matches_apply_token(golden):
    """ApplyToken readout with key = 0, decay = 1 (capsule.cpp:281-304, 354-397)."""
    g = golden["heads"]
    got = oracle.project(g["codes"], g["smoothing"], g["scales"], g["query"],
                         g["compensator_keys"], g["compensator_values"])
    np.testing.assert_allclose(got, g["projection"], rtol=1e-5, atol=1e-6)
    assert_same_bits("ApplyToken readout", got, g["projection"])


def test_oracle_small_state_matches_reference(golden):
    """The reference test's own 8x6 state (capsule_test.cpp:40-48): the oracle
    handles any geometry, not only 128x128."""
    s = golden["small"]
    residual = oracle.rebuild_residual(s["dense"], s["compensator_keys"], s["compensator_values"])
    z, c, b = oracle.quantize(residual[None], "capsule")
    assert_same_bits("codes", z[0], s["codes"])
    assert_same_bits("smoothing", c[0], s["smoothing"])
    assert_same_bits("scales", b[0], s["scales"])
    dense = oracle.dequantize(s["codes"][None], s["smoothing"][None], s["scales"][None],
                              s["compensator_keys"][None], s["compensator_values"][None])
    assert_same_bits("DenseState", dense[0], s["dense_state"])
    out = oracle.project(s["codes"][None], s["smoothing"][None], s["scales"][None],
                         s["query"][None], s["compensator_keys"][None],
                         s["compensator_values"][None])
    assert_same_bits("ApplyToken readout", out[0], s["projection"])


def test_adapter_transpose_vector(golden):
    """Provider [value, key] -> capsule [key, value]: the reference adapter
    test's vector {1,4,2,5,3,6} (qwen38_gdn_adapter_test.cpp:20-31)."""
    a = golden["adapter"]
    np.testing.assert_array_equal(a["capsule"].ravel(), [1, 4, 2, 5, 3, 6])
    np.testing.assert_array_equal(oracle.provider_to_capsule(a["provider"][None])[0], a["capsule"])
    np.testing.assert_array_equal(oracle.capsule_to_provider(a["capsule"][None])[0], a["provider"])


def test_provider_layout_is_the_transpose():
    """Provider-layout quantize / dequantize / projection equal the capsule
    results on the transposed head (smoothing per key, scales per value)."""
    rng = np.random.default_rng(11)
    cap = (rng.standard_normal((6, 128, 128)) * 10.0 ** -rng.uniform(0, 3, (6, 1, 1))
           ).astype(np.float32)
    cap[rng.random(cap.shape) < 0.01] = 0.0
    prov = np.ascontiguousarray(cap.transpose(0, 2, 1))
    zc, cc, bc = oracle.quantize(cap, "capsule")
    zp, cp, bp = oracle.quantize(prov, "provider")
    assert_same_bits("codes", zp, zc.transpose(0, 2, 1))
    assert_same_bits("smoothing", cp, cc)
    assert_same_bits("scales", bp, bc)
    dc = oracle.dequantize(zc, cc, bc, layout="capsule")
    dp = oracle.dequantize(zp, cp, bp, layout="provider")
    assert_same_bits("dense", dp, dc.transpose(0, 2, 1))
    q = rng.standard_normal((6, 128)).astype(np.float32)
    assert_same_bits("projection", oracle.project(zp, cp, bp, q, layout="provider"),
                     oracle.project(zc, cc, bc, q, layout="capsule"))


def test_two_stage_equals_fused():
    rng = np.random.default_rng(5)
    state = rng.standard_normal((4, 128, 128)).astype(np.float32)
    for layout in ("capsule", "provider"):
        z, c, b = oracle.quantize(state, layout)
        c2 = oracle.smoothing(state, layout)
        z2, _, b2 = oracle.quantize(state, layout, smoothing_in=c2)
        assert_same_bits("smoothing", c2, c)
        assert_same_bits("codes", z2, z)
        assert_same_bits("scales", b2, b)


def test_sign_of_zero_does_not_reach_the_int8_stage():
    """The window refit may turn a -0 of DenseState into +0 (its products are
    formed as fma(a, b, +0)); quantizing either gives the same codes,
    smoothing and scales, so the boundary it writes is unchanged."""
    rng = np.random.default_rng(11)
    state = rng.standard_normal((2, 128, 128)).astype(np.float32)
    state[rng.random(state.shape) < 0.05] = 0.0
    flipped = state.copy()
    zeros = flipped == 0.0
    flipped[zeros] = np.float32(-0.0)
    assert np.signbit(flipped[zeros]).all() and not np.signbit(state[zeros]).any()
    for layout in ("capsule", "provider"):
        for got, want, what in zip(oracle.quantize(flipped, layout), oracle.quantize(state, layout),
                                   ("codes", "smoothing", "scales")):
            assert_same_bits(what, got, want)


def test_quant_only_semantics_by_hand():
    """A head worked out by hand from capsule.cpp:190-225: zero columns give
    scale 0 and codes 0; the largest magnitude per value gets code +-127."""
    state = np.zeros((1, 128, 128), np.float32)
    state[0, 3, 5] = -2.0
    state[0, 3, 6] = 1.0
    state[0, 9, 5] = 0.5
    z, c, b = oracle.quantize(state, "capsule")
    c3 = np.float32(np.sqrt(np.float32(3.0 / 128.0)))
    c9 = np.float32(np.sqrt(np.float32(0.5 / 128.0)))
    assert c[0, 3] == c3 and c[0, 9] == c9
    assert c[0, 0] == np.float32(np.sqrt(np.float32(1e-8)))
    assert b[0, 5] == max(np.float32(2.0) / c3, np.float32(0.5) / c9)
    assert b[0, 6] == np.float32(1.0) / c3
    assert (b[0, [0, 1, 2, 7]] == 0).all()
    assert abs(int(z[0, 3, 6])) == 127 and int(z[0, 3, 6]) > 0
    assert int(np.abs(z[0, :, 5]).max()) == 127
    nonzero = {(3, 5), (3, 6), (9, 5)}
    mask = np.ones((128, 128), bool)
    for k, v in nonzero:
        mask[k, v] = False
    assert (z[0][mask] == 0).all()


def test_oracle_matches_reference_quant_only_fixture(golden):
    """The reference's own quant-only stage (QuantizeBoundary /
    DequantizeBoundary / ReadWindowState at rank 0) on benchmark heads and
    edge cases: zero head, zero row and column, denormals, 1e-30..1e30
    range, rounding ties, dyadic grid."""
    g = golden["quant_only"]
    z, c, b = oracle.quantize(g["states"], "capsule")
    assert_same_bits("codes", z, g["codes"])
    assert_same_bits("smoothing", c, g["smoothing"])
    assert_same_bits("scales", b, g["scales"])
    assert_same_bits("dense", oracle.dequantize(z, c, b), g["dense"])
    assert_same_bits("projection", oracle.project(z, c, b, g["query"]), g["projection"])


# ---------------------------------------------------------------------------
# Against the reference library compiled in this container (oracle/_ref).

need_ref = pytest.mark.skipif(not oracle.ref_available(),
                              reason="reference library not built (make -C oracle ref)")


def _benchmark_head(rng: np.random.Generator) -> np.ndarray:
    head = (rng.standard_normal((128, 128)) * 10.0 ** (-3.0 * rng.random())).astype(np.float32)
    head[rng.random((128, 128)) < 0.01] = 0.0
    return head


@need_ref
@pytest.mark.parametrize("case", ["benchmark", "wide", "holes", "tiny", "ties"])
def test_oracle_vs_reference_library(case):
    """Fresh heads through the reference's FromDenseBoundary: the oracle,
    given the reference's residual, reproduces codes, smoothing, scales,
    DenseState and the ApplyToken readout."""
    seeds = {"benchmark": 101, "wide": 102, "holes": 103, "tiny": 104, "ties": 105}
    rng = np.random.default_rng(seeds[case])
    if case == "benchmark":
        head = _benchmark_head(rng)
    elif case == "wide":
        head = (rng.standard_normal((128, 128)) * 10.0 ** rng.uniform(-8, 4, (128, 1))
                ).astype(np.float32)
    elif case == "holes":
        head = _benchmark_head(rng)
        head[40, :] = 0.0
        head[:, 7] = 0.0
    elif case == "tiny":
        head = (rng.standard_normal((128, 128)) * 1e-20).astype(np.float32)
    else:
        head = (rng.integers(-64, 65, (128, 128)) * 2.0 ** -7).astype(np.float32)
    q = rng.standard_normal(128).astype(np.float32)
    q /= np.float32(np.linalg.norm(q))
    r = oracle.ref_codec_head(head, q)
    residual = oracle.rebuild_residual(head, r["compensator_keys"], r["compensator_values"])
    z, c, b = oracle.quantize(residual[None], "capsule")
    assert_same_bits("codes", z[0], r["codes"])
    assert_same_bits("smoothing", c[0], r["smoothing"])
    assert_same_bits("scales", b[0], r["scales"])
    dense = oracle.dequantize(z, c, b, r["compensator_keys"][None], r["compensator_values"][None])
    assert_same_bits("DenseState", dense[0], r["dense_state"])
    out = oracle.project(z, c, b, q[None], r["compensator_keys"][None],
                         r["compensator_values"][None])
    assert_same_bits("ApplyToken readout", out[0], r["projection"])


@need_ref
@pytest.mark.parametrize("program", ["sha256_test", "gdn_state_codec_state_capsule_test",
                                     "gdn_state_codec_qwen38_gdn_adapter_test"])
def test_reference_own_tests_pass(program):
    """The reference's ctest programs (CMakeLists.txt:19-26), compiled from its
    sources by oracle/Makefile, pass on this build of its library."""
    path = oracle.ORACLE_DIR / "_ref" / program
    if not path.is_file():
        pytest.skip(f"{program} not built")
    result = subprocess.run([str(path)], capture_output=True, text=True, timeout=120)
    assert result.returncode == 0, result.stdout + result.stderr


need_ref_quant = pytest.mark.skipif(not oracle.ref_quant_available(),
                                    reason="reference quant-only library not built")


@need_ref_quant
def test_oracle_vs_reference_quant_only_stage():
    """512 fresh heads of the benchmark distribution and 64 wide-range heads
    through the reference's own quant-only code: identical bits everywhere."""
    rng = np.random.default_rng(2024)
    heads = np.stack([_benchmark_head(rng) for _ in range(512)])
    wide = (rng.standard_normal((64, 128, 128)) * 10.0 ** rng.uniform(-20, 20, (64, 128, 1))
            ).astype(np.float32)
    for states in (heads, wide):
        z, c, b = oracle.quantize(states, "capsule", threads=4)
        rz, rc, rb = oracle.ref_quant_encode(states, threads=4)
        assert_same_bits("codes", z, rz)
        assert_same_bits("smoothing", c, rc)
        assert_same_bits("scales", b, rb)
        assert_same_bits("dense", oracle.dequantize(z, c, b, threads=4),
                         oracle.ref_quant_decode(rz, rc, rb, threads=4))
        q = rng.standard_normal((states.shape[0], 128)).astype(np.float32)
        assert_same_bits("projection", oracle.project(z, c, b, q, threads=4),
                         oracle.ref_quant_project(rz, rc, rb, q, threads=4))


@need_ref_quant
def test_oracle_vs_reference_quant_only_property():
    """Property check against the reference's own quant-only code over
    generated heads: per-row and per-column magnitudes spread over up to 60
    decades, sparse heads, signed zeros, exact dyadic values and repeated
    magnitudes (rounding ties)."""
    hypothesis = pytest.importorskip("hypothesis")
    st = hypothesis.strategies

    @hypothesis.settings(max_examples=40, deadline=None, derandomize=True)
    @hypothesis.given(seed=st.integers(0, 2**32 - 1),
                      row_decades=st.floats(0.0, 30.0), col_decades=st.floats(0.0, 30.0),
                      zero_fraction=st.sampled_from([0.0, 0.01, 0.5, 0.99]),
                      kind=st.sampled_from(["normal", "dyadic", "repeated"]),
                      negative_zeros=st.booleans())
    def check(seed, row_decades, col_decades, zero_fraction, kind, negative_zeros):
        rng = np.random.default_rng(seed)
        if kind == "normal":
            head = rng.standard_normal((128, 128))
        elif kind == "dyadic":
            head = rng.integers(-255, 256, (128, 128)) * 2.0 ** -8
        else:
            head = rng.choice([-1.5, -0.75, 0.75, 1.5, 3.0], (128, 128))
        head = head * 10.0 ** (row_decades * (rng.random((128, 1)) - 0.5))
        head = head * 10.0 ** (col_decades * (rng.random((1, 128)) - 0.5))
        head = head.astype(np.float32)
        head[rng.random((128, 128)) < zero_fraction] = np.float32(-0.0 if negative_zeros else 0.0)
        states = head[None]
        z, c, b = oracle.quantize(states, "capsule")
        rz, rc, rb = oracle.ref_quant_encode(states)
        assert_same_bits("codes", z, rz)
        assert_same_bits("smoothing", c, rc)
        assert_same_bits("scales", b, rb)
        assert_same_bits("dense", oracle.dequantize(z, c, b), oracle.ref_quant_decode(rz, rc, rb))

    check()
