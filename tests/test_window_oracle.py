"""CPU tests of the windowed-decode oracle (oracle/gdn_window_oracle.c).

The oracle is pinned to the reference library itself: its window read
against ReadWindowState (capsule.cpp:256-304, through ref_quant_shim.cpp),
its token sequence against ApplyToken (capsule.cpp:354-397, through
ref_shim.cpp) including the window refits, and its boundary fit against
FromDenseBoundary -- all bit for bit with fp32 record storage.  With the
device ABI's binary16 storage it then has to pass the reference's own window
probe gates (relative RMS against the dense fp32 step)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
import window_cases as wc

ref_only = pytest.mark.skipif(not oracle.ref_available(), reason="reference library not built")
ref_quant_only = pytest.mark.skipif(not oracle.ref_quant_available(),
                                    reason="reference quant-only library not built")


def bits(x):
    return np.ascontiguousarray(x, np.float32).view(np.uint32)


def test_binary16_rounding_matches_numpy():
    rng = np.random.default_rng(3)
    x = (rng.standard_normal(20000) * 10.0 ** rng.integers(-9, 6, 20000)).astype(np.float32)
    x = np.concatenate([x, np.array([65504, 65519.99, 65520, 1e6, 5.96e-8, 2.98e-8, 2.99e-8,
                                     6.1e-5, 6.09e-5, -0.0, 0.0, np.inf, -np.inf], np.float32)])
    with np.errstate(over="ignore"):
        want = x.astype(np.float16).view(np.uint16)
    got = np.array([oracle.f32_to_f16_bits(v) for v in x], np.uint16)
    assert np.array_equal(got, want)


def test_bfloat16_rounding_matches_torch():
    rng = np.random.default_rng(4)
    x = (rng.standard_normal(20000) * 10.0 ** rng.integers(-30, 30, 20000)).astype(np.float32)
    want = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(oracle.f32_to_bf16_array(x), want)
    assert all(oracle.f32_to_bf16_bits(v) == w for v, w in zip(x[:500], want[:500]))


def _random_head(rng, position: int, compensators: bool) -> oracle.WindowHead:
    dense = (rng.standard_normal((128, 128)) * 0.2).astype(np.float32)
    z, c, b = oracle.quantize(dense[None], "capsule")
    ck = wc.f16(rng.standard_normal((128, 4)) * 0.05) if compensators else None
    cv = wc.f16(rng.standard_normal((128, 4)) * 0.05) if compensators else None
    h = oracle.WindowHead(z[0], c[0], b[0], ck, cv, layout="capsule")
    h.rdecay[:position] = (0.9 + 0.1 * rng.random(position)).astype(np.float32)
    h.rkeys[:position] = wc.f16(rng.standard_normal((position, 128)) * 0.1)
    h.rcorr[:position] = wc.f16(rng.standard_normal((position, 128)))
    h.position.value = position
    return h


@ref_quant_only
@pytest.mark.parametrize("position", [0, 1, 7, 15, 16])
@pytest.mark.parametrize("compensators", [False, True])
def test_window_read_matches_reference(position, compensators):
    rng = np.random.default_rng(100 + position + 50 * compensators)
    h = _random_head(rng, position, compensators)
    x = rng.standard_normal(128).astype(np.float32)
    assert np.array_equal(bits(h.read(x)), bits(oracle.ref_window_read(h, x)))


def _token_stream(rng, tokens):
    decay = (0.9 + 0.09 * rng.random(tokens)).astype(np.float32)
    k = rng.standard_normal((tokens, 128)).astype(np.float32)
    k /= np.linalg.norm(k, axis=1, keepdims=True)
    beta = rng.random(tokens).astype(np.float32)
    key = (beta[:, None] * k).astype(np.float32)
    read = (decay[:, None] * k).astype(np.float32)
    query = (rng.standard_normal((tokens, 128)) * 0.088).astype(np.float32)
    value = rng.standard_normal((tokens, 128)).astype(np.float32)
    return decay, key, read, query, value


@ref_only
@pytest.mark.parametrize("seed", [5, 6])
def test_token_sequence_matches_reference_apply_token(seed):
    """40 tokens (two window refits) from FromDenseBoundary: outputs and the
    final DenseState bit-identical to the reference with fp32 storage."""
    rng = np.random.default_rng(seed)
    dense = (rng.standard_normal((128, 128)) * 0.3).astype(np.float32)
    tokens = 40
    decay, key, read, query, value = _token_stream(rng, tokens)
    ref = oracle.ref_apply_tokens(dense, decay, key, read, query, value)
    assert list(np.nonzero(ref["crossed"])[0]) == [15, 31]
    b = oracle.quantize_boundary(dense, 32, "capsule")
    h = oracle.WindowHead(b["codes"], b["smoothing"], b["scales"], b["compensator_keys"],
                          b["compensator_values"], layout="capsule")
    outs = []
    for t in range(tokens):
        outs.append(h.step(decay[t], key[t], read[t], query[t], value[t], round_storage=False))
        if h.position.value == wc.WINDOW:
            assert h.fold(32, round_storage=False) == 0
    assert np.array_equal(bits(np.array(outs)), bits(ref["outputs"]))
    assert h.position.value == ref["position"] == 8
    assert np.array_equal(bits(h.dense()), bits(ref["dense"]))


@ref_only
def test_boundary_fit_matches_reference():
    rng = np.random.default_rng(8)
    for scale in (1.0, 1e-3):
        dense = (rng.standard_normal((128, 128)) * scale).astype(np.float32)
        got = oracle.quantize_boundary(dense, 32, "capsule")
        want = oracle.ref_codec_head(dense)
        assert got["status"] == 0
        assert np.array_equal(got["codes"], want["codes"])
        for name in ("smoothing", "scales", "compensator_keys", "compensator_values"):
            assert np.array_equal(bits(got[name]), bits(want[name])), name


def test_quant_only_boundary_is_the_int8_stage():
    rng = np.random.default_rng(9)
    dense = (rng.standard_normal((128, 128)) * 0.01).astype(np.float32)
    got = oracle.quantize_boundary(dense, 0, "provider")
    z, c, b = oracle.quantize(np.ascontiguousarray(dense.T)[None], "provider")
    assert np.array_equal(got["codes"], z[0])
    assert np.array_equal(bits(got["smoothing"]), bits(c[0]))
    assert np.array_equal(bits(got["scales"]), bits(b[0]))
    assert not got["compensator_keys"].any() and not got["compensator_values"].any()


def test_step_probe_gate_with_binary16_records():
    """The reference's windowed-step probe gate (output and state relative RMS
    below 0.0025 against the dense fp32 step) on the oracle's generic step."""
    case = wc.step_probe_case(states=8)
    heads = wc.window_heads(case, "capsule")
    outs, dense_outs, window_dense, dense_after = [], [], [], []
    for st, h in enumerate(heads):
        state = h.dense()  # the window's dense state before the token
        outs.append(h.step(case["decay"][st], case["write_keys"][st], case["reads"][st],
                           case["queries"][st], case["values"][st], round_storage=True))
        dense_outs.append(oracle.dense_step(state, case["decay"][st], case["write_keys"][st],
                                            case["reads"][st], case["queries"][st],
                                            case["values"][st]))
        window_dense.append(h.dense())
        dense_after.append(state)
        assert h.position.value == case["position"] + 1
    assert wc.relative_rms(outs, dense_outs) < 0.0025
    assert wc.relative_rms(window_dense, dense_after) < 0.0025


def test_boundary_probe_gate():
    """The reference's refit probe gate: quant-only refit within 2e-2 relative
    RMS of the window's dense state, the power-iteration refit better than
    the compensator-free requantization, and the window cleared."""
    case = wc.boundary_probe_case(states=4)
    for iterations in (0, 32):
        errors, plain = [], []
        for h in wc.window_heads(case, "provider"):
            before = h.dense()
            assert h.fold(iterations, round_storage=True) == 0
            assert h.position.value == 0
            assert not h.rdecay.any() and not h.rkeys.any() and not h.rcorr.any()
            errors.append(wc.relative_rms(h.dense(), before))
            q = oracle.quantize_boundary(before, 0, "capsule")
            requant = oracle.WindowHead(q["codes"], q["smoothing"], q["scales"],
                                        layout="capsule").dense()
            plain.append(wc.relative_rms(requant, before))
        if iterations == 0:
            assert max(errors) < 2e-2
        else:
            assert max(e - p for e, p in zip(errors, plain)) < 0
