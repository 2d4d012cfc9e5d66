"""Input cases for the windowed decode tests (CPU and GPU).

``step_probe_case`` and ``boundary_probe_case`` rebuild, from their
formulas, the fixtures of the reference's own window probes (native/ascendc/
gdn_state_codec/host/gdn_state_codec_windowed_gdn_runtime_probe.cpp:187-234
and gdn_state_codec_window_boundary_runtime_probe.cpp:197-236), whose gates
the tests apply: output and state relative RMS < 0.0025 against the dense
fp32 step, and a refit within 2e-2 relative RMS (quant-only) or better than
the compensator-free requantization (power iterations).  ``qwen_case`` is a
seeded Qwen3.5-style decode token stream over a real INT8 boundary.

binary16 values are numpy float16 (round to nearest even, like the probes'
aclFloatToFloat16); they are carried here as float32 arrays holding exactly
representable values, plus the raw bits for the device buffers.
"""

from __future__ import annotations

import numpy as np

import oracle

D, RANK, WINDOW, STRIDE = 128, 4, 16, 8


def f16(x) -> np.ndarray:
    """Round to binary16 and back (float32 array of representable values)."""
    return np.asarray(x, np.float32).astype(np.float16).astype(np.float32)


def f16_bits(x) -> np.ndarray:
    return np.asarray(x, np.float32).astype(np.float16).view(np.uint16)


def _fsin(x) -> np.ndarray:
    return np.sin(np.asarray(x, np.float32)).astype(np.float32)


def _fcos(x) -> np.ndarray:
    return np.cos(np.asarray(x, np.float32)).astype(np.float32)


def _boundary_formulas(states: int) -> dict:
    s = np.arange(states)[:, None]
    a = np.arange(D)[None, :]
    smoothing = (np.float32(0.75) + np.float32(0.002) * ((s + a) % 41).astype(np.float32))
    scales = (np.float32(0.11) + np.float32(0.001) * ((3 * s + a) % 29).astype(np.float32))
    r = np.arange(RANK)[None, None, :]
    sa = (s + a)[:, :, None]
    ck = f16(np.float32(0.008) * _fsin((sa + r + 1).astype(np.float32) * np.float32(0.071)))
    cv = f16(np.float32(0.009) * _fcos((sa + r + 2).astype(np.float32) * np.float32(0.067)))
    index = np.arange(D * D)[None, :]
    codes = (((index * 17 + s * 11) % 255) - 127).astype(np.int8).reshape(states, D, D)
    return {"codes": codes, "smoothing": smoothing.astype(np.float32),
            "scales": scales.astype(np.float32), "ck": ck, "cv": cv}


def _records(states: int, position: int) -> dict:
    decay = np.zeros((states, WINDOW), np.float32)
    keys = np.zeros((states, WINDOW, D), np.float32)
    corr = np.zeros((states, WINDOW, D), np.float32)
    for st in range(states):
        for rec in range(position):
            decay[st, rec] = np.float32(0.93) + np.float32(0.002) * np.float32((st + rec) % 9)
            base = (st * WINDOW + rec) * D
            axis = np.arange(D)
            keys[st, rec] = f16(np.float32(0.026) * _fsin((base + axis + 1).astype(np.float32)
                                                          * np.float32(0.007)))
            corr[st, rec] = f16(np.float32(0.082) * _fcos((base + axis + 1).astype(np.float32)
                                                          * np.float32(0.005)))
    return {"record_decay": decay, "record_keys": keys, "record_corrections": corr,
            "position": position}


def step_probe_case(states: int = 32, position: int = 7) -> dict:
    """The windowed runtime probe's inputs (generic step, codes [key][value])."""
    case = _boundary_formulas(states)
    case.update(_records(states, position))
    s = np.arange(states)[:, None]
    a = np.arange(D)[None, :]
    flat = (s * D + a).astype(np.float32)
    case["decay"] = (np.float32(0.94) + np.float32(0.001) * (np.arange(states) % 7)).astype(
        np.float32)
    case["write_keys"] = f16(np.float32(0.035) * _fsin((flat + 1) * np.float32(0.013)))
    case["reads"] = f16(np.float32(0.031) * _fcos((flat + 3) * np.float32(0.017)))
    case["queries"] = f16(np.float32(0.029) * _fsin((flat + 5) * np.float32(0.019)))
    case["values"] = f16(np.float32(0.12) * _fcos((flat + 7) * np.float32(0.011)))
    return case


def boundary_probe_case(states: int = 32) -> dict:
    """The boundary refit probe's inputs (full windows)."""
    case = _boundary_formulas(states)
    case.update(_records(states, WINDOW))
    return case


def window_heads(case: dict, layout: str, compensators: bool = True) -> list:
    """oracle.WindowHead per state of a probe case (codes given as [key][value]
    and transposed for the provider layout)."""
    heads = []
    for st in range(case["codes"].shape[0]):
        codes = case["codes"][st]
        if layout == "provider":
            codes = np.ascontiguousarray(codes.T)
        h = oracle.WindowHead(codes, case["smoothing"][st], case["scales"][st],
                              case["ck"][st] if compensators else None,
                              case["cv"][st] if compensators else None, layout=layout)
        p = case["position"]
        h.rdecay[:p] = case["record_decay"][st, :p]
        h.rkeys[:p] = case["record_keys"][st, :p]
        h.rcorr[:p] = case["record_corrections"][st, :p]
        h.position.value = p
        heads.append(h)
    return heads


def relative_rms(actual, reference) -> float:
    actual = np.asarray(actual, np.float64)
    reference = np.asarray(reference, np.float64)
    return float(np.sqrt(((actual - reference) ** 2).sum() / max((reference ** 2).sum(), 1e-30)))


def qwen_tokens(heads: int, tokens: int, seed: int) -> dict:
    """Seeded Qwen3.5 decode inputs for `tokens` steps of `heads` value heads:
    log decay in [-0.1, -0.005], beta in (0, 1), unit-norm bf16 q / k for
    heads/2 query-key heads, N(0, 1) bf16 values."""
    rng = np.random.default_rng(seed)
    log_decay = -(0.005 + 0.095 * rng.random((tokens, heads))).astype(np.float32)
    beta = oracle.f32_to_bf16_array(rng.random((tokens, heads)).astype(np.float32))
    k = rng.standard_normal((tokens, heads // 2, D)).astype(np.float32)
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    q = rng.standard_normal((tokens, heads // 2, D)).astype(np.float32)
    q /= np.linalg.norm(q, axis=-1, keepdims=True)
    v = rng.standard_normal((tokens, heads, D)).astype(np.float32)
    return {"log_decay": log_decay, "beta": beta,
            "keys": oracle.f32_to_bf16_array(k), "queries": oracle.f32_to_bf16_array(q),
            "values": oracle.f32_to_bf16_array(v)}
