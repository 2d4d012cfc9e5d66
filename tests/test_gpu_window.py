"""GPU tests of the windowed decode kernels against the CPU oracle
(oracle/gdn_window_oracle.c, itself pinned to the reference library's
ReadWindowState / ApplyToken / FromDenseBoundary): outputs, appended records,
positions and refit boundaries bit for bit, with the ABI's binary16 record
and compensator storage; plus the reference window probes' RMS gates."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
import window_cases as wc
from gdn_state_codec import _native, codec
from gdn_state_codec import runtime as runtime_mod
from gdn_state_codec.config import GdnStateCodecExperiment

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def bits(x):
    return np.ascontiguousarray(x, np.float32).view(np.uint32)


def f16_dev(x) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(wc.f16_bits(x))).view(torch.float16).to(DEV)


def bf16_dev(bits16) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits16)).view(torch.bfloat16).to(DEV)


def f32_dev(x) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(x, np.float32)).to(DEV)


def bf16_dev_shifted(bits16) -> torch.Tensor:
    """The same bf16 values one element past an aligned address: rows only
    2-byte aligned, which the staged step cannot copy, so the launch takes
    the unstaged kernel."""
    host = torch.from_numpy(np.ascontiguousarray(bits16)).view(torch.bfloat16)
    buf = torch.empty(host.numel() + 1, dtype=torch.bfloat16, device=DEV)
    view = buf[1:].view(host.shape)
    view.copy_(host)
    assert view.data_ptr() % 16 == 2
    return view


def window_from_case(case, layout, compensators=True) -> codec.WindowStates:
    codes = case["codes"] if layout == "capsule" else np.ascontiguousarray(
        case["codes"].transpose(0, 2, 1))
    enc = codec.EncodedStates(torch.from_numpy(codes).to(DEV), f32_dev(case["smoothing"]),
                              f32_dev(case["scales"]), layout)
    w = codec.new_window(enc, f16_dev(case["ck"]) if compensators else None,
                         f16_dev(case["cv"]) if compensators else None)
    w.record_decay.copy_(f32_dev(case["record_decay"]))
    w.record_keys.copy_(f16_dev(case["record_keys"]))
    w.record_corrections.copy_(f16_dev(case["record_corrections"]))
    w.positions[:, 0] = case["position"]
    return w


def check_records(window, heads, what=""):
    torch.cuda.synchronize()
    rk = window.record_keys.float().cpu().numpy()
    rc = window.record_corrections.float().cpu().numpy()
    rd = window.record_decay.cpu().numpy()
    pos = window.positions[:, 0].cpu().numpy()
    for i, h in enumerate(heads):
        assert pos[i] == h.position.value, f"{what} head {i} position"
        assert np.array_equal(bits(rk[i]), bits(h.rkeys)), f"{what} head {i} record keys"
        assert np.array_equal(bits(rc[i]), bits(h.rcorr)), f"{what} head {i} record corrections"
        p = h.position.value
        assert np.array_equal(bits(rd[i, :p]), bits(h.rdecay[:p])), f"{what} head {i} decays"


def test_generic_step_matches_oracle_and_passes_the_probe_gate():
    case = wc.step_probe_case(states=32)
    window = window_from_case(case, "capsule")
    heads = wc.window_heads(case, "capsule")
    dense_before = np.stack([h.dense() for h in heads])
    out = codec.window_step(window, f32_dev(case["decay"]), f16_dev(case["write_keys"]),
                            f16_dev(case["reads"]), f16_dev(case["queries"]),
                            f16_dev(case["values"]))
    want = np.stack([h.step(case["decay"][i], case["write_keys"][i], case["reads"][i],
                            case["queries"][i], case["values"][i]) for i, h in enumerate(heads)])
    assert np.array_equal(bits(out.cpu().numpy()), bits(want))
    check_records(window, heads, "generic")
    # the dense fp32 step from the same state (fp32_gdn_step_launch_v1)
    dense = f32_dev(dense_before)
    dense_out = codec.dense_step(dense, f32_dev(case["decay"]), f16_dev(case["write_keys"]),
                                 f16_dev(case["reads"]), f16_dev(case["queries"]),
                                 f16_dev(case["values"]))
    host = dense_before.copy()
    want_dense = np.stack([oracle.dense_step(host[i], case["decay"][i], case["write_keys"][i],
                                             case["reads"][i], case["queries"][i],
                                             case["values"][i]) for i in range(32)])
    assert np.array_equal(bits(dense_out.cpu().numpy()), bits(want_dense))
    assert np.array_equal(bits(dense.cpu().numpy()), bits(host))
    # the reference probe's gate
    assert wc.relative_rms(out.cpu().numpy(), want_dense) < 0.0025
    window_dense = np.stack([h.dense() for h in heads])
    assert wc.relative_rms(window_dense, host) < 0.0025


def _qwen_boundary(heads, full, seed):
    states = codec.synthesize_states(1, 1, heads, layout="provider", seed=seed, device=DEV)
    states = states.reshape(heads, 128, 128)
    if full:
        enc = codec.full_encode(states, "provider")
        ck = enc.compensator_keys.half().contiguous()
        cv = enc.compensator_values.half().contiguous()
        return codec.new_window(enc.encoded, ck, cv)
    return codec.new_window(codec.quantize(states, "provider"))


def _oracle_heads(window):
    torch.cuda.synchronize()
    enc = window.encoded
    codes, c, b = enc.codes.cpu().numpy(), enc.smoothing.cpu().numpy(), enc.scales.cpu().numpy()
    ck = None if window.compensator_keys is None else window.compensator_keys.float().cpu().numpy()
    cv = None if window.compensator_values is None else window.compensator_values.float().cpu().numpy()
    heads = []
    for i in range(codes.shape[0]):
        h = oracle.WindowHead(codes[i], c[i], b[i], None if ck is None else ck[i],
                              None if cv is None else cv[i], layout="provider")
        heads.append(h)
    return heads


def _assert_boundary(window, heads, what):
    torch.cuda.synchronize()
    enc = window.encoded
    codes = enc.codes.cpu().numpy()
    c, b = enc.smoothing.cpu().numpy(), enc.scales.cpu().numpy()
    for i, h in enumerate(heads):
        assert np.array_equal(codes[i], h.codes), f"{what} head {i} codes"
        assert np.array_equal(bits(c[i]), bits(h.c)), f"{what} head {i} smoothing"
        assert np.array_equal(bits(b[i]), bits(h.b)), f"{what} head {i} scales"
        if h.ck is not None:
            ck = window.compensator_keys[i].float().cpu().numpy()
            cv = window.compensator_values[i].float().cpu().numpy()
            assert np.array_equal(bits(ck), bits(h.ck)), f"{what} head {i} compensator keys"
            assert np.array_equal(bits(cv), bits(h.cv)), f"{what} head {i} compensator values"


@pytest.mark.parametrize("full, iterations, staged", [(False, 0, True), (True, 32, True),
                                                      (True, 4, True), (False, 0, False),
                                                      (True, 4, False)])
def test_qwen_decode_sequence_with_refit_matches_oracle(full, iterations, staged):
    """20 Qwen3.5 tokens over 16 value heads: bf16 outputs, records and the
    refit boundary after token 16 bit-identical to the oracle.  `staged`:
    16-byte aligned token rows (the staged step kernel); otherwise rows only
    2-byte aligned (the unstaged kernel)."""
    nheads, tokens = 16, 20
    tok = bf16_dev if staged else bf16_dev_shifted
    window = _qwen_boundary(nheads, full, seed=31 + iterations)
    heads = _oracle_heads(window)
    if not full:
        for h in heads:
            h.ck = h.cv = None
    inputs = wc.qwen_tokens(nheads, tokens, seed=7 + iterations)
    for t in range(tokens):
        if t == wc.WINDOW:
            window = codec.window_refit(window, iterations)
            for h in heads:
                assert h.fold(iterations, round_storage=True) == 0
            _assert_boundary(window, heads, f"refit ({iterations} iterations)")
            check_records(window, heads, "after refit")
        out = codec.window_step_bf16(window, f32_dev(inputs["log_decay"][t]),
                                     tok(inputs["beta"][t]), tok(inputs["keys"][t]),
                                     tok(inputs["queries"][t]), tok(inputs["values"][t]))
        torch.cuda.synchronize()
        pos = heads[0].position.value
        alpha = window.record_decay[:, pos].cpu().numpy()
        # the device's exp is within 2 ulp of the correctly rounded exp
        exact = np.exp(inputs["log_decay"][t].astype(np.float64)).astype(np.float32)
        assert np.all(np.abs(bits(alpha).astype(np.int64) - bits(exact).astype(np.int64)) <= 2)
        want = []
        for i, h in enumerate(heads):
            token = oracle.qwen_token(alpha[i], inputs["beta"][t][i], inputs["keys"][t][i // 2],
                                      inputs["queries"][t][i // 2], inputs["values"][t][i])
            want.append(h.step(*token, round_storage=True))
        got = out.view(torch.int16).cpu().numpy().view(np.uint16)
        assert np.array_equal(got, oracle.f32_to_bf16_array(np.stack(want))), f"token {t}"
        check_records(window, heads, f"token {t}")


@pytest.mark.parametrize("full", [False, True])
def test_decode_and_refit_with_more_heads_than_resident_ctas(full):
    """1,536 value heads (more than the 592 CTAs a B200 keeps resident), so
    every CTA of the staged step and of the pipelined quant-only refit takes
    several heads through its one-ahead stage: 18 tokens with a refit after
    token 16, a seeded sample of 40 heads (both halves of the range) checked
    bit for bit against the oracle, and every head's record state against the
    sampled heads' oracle at the end."""
    nheads, tokens = 1536, 18
    window = _qwen_boundary(nheads, full, seed=91)
    rng = np.random.default_rng(92)
    sample = np.sort(np.concatenate([rng.choice(592, 20, replace=False),
                                     592 + rng.choice(nheads - 592, 20, replace=False)]))
    torch.cuda.synchronize()
    enc = window.encoded
    codes = enc.codes.cpu().numpy()
    c, b = enc.smoothing.cpu().numpy(), enc.scales.cpu().numpy()
    ck = None if not full else window.compensator_keys.float().cpu().numpy()
    cv = None if not full else window.compensator_values.float().cpu().numpy()
    heads = {int(i): oracle.WindowHead(codes[i], c[i], b[i], None if ck is None else ck[i],
                                       None if cv is None else cv[i], layout="provider")
             for i in sample}
    inputs = wc.qwen_tokens(nheads, tokens, seed=93)
    for t in range(tokens):
        if t == wc.WINDOW:
            window = codec.window_refit(window, 0)
            torch.cuda.synchronize()
            nz = window.encoded.codes.cpu().numpy()
            nc = window.encoded.smoothing.cpu().numpy()
            nb = window.encoded.scales.cpu().numpy()
            for i, h in heads.items():
                assert h.fold(0, round_storage=True) == 0
                assert np.array_equal(nz[i], h.codes), f"refit head {i} codes"
                assert np.array_equal(bits(nc[i]), bits(h.c)), f"refit head {i} smoothing"
                assert np.array_equal(bits(nb[i]), bits(h.b)), f"refit head {i} scales"
        out = codec.window_step_bf16(window, f32_dev(inputs["log_decay"][t]),
                                     bf16_dev(inputs["beta"][t]), bf16_dev(inputs["keys"][t]),
                                     bf16_dev(inputs["queries"][t]), bf16_dev(inputs["values"][t]))
        torch.cuda.synchronize()
        got = out.view(torch.int16).cpu().numpy().view(np.uint16)
        pos = next(iter(heads.values())).position.value
        alpha = window.record_decay[:, pos].cpu().numpy()
        for i, h in heads.items():
            token = oracle.qwen_token(alpha[i], inputs["beta"][t][i], inputs["keys"][t][i // 2],
                                      inputs["queries"][t][i // 2], inputs["values"][t][i])
            want = h.step(*token, round_storage=True)
            assert np.array_equal(got[i], oracle.f32_to_bf16_array(want[None])[0]), \
                f"token {t} head {i}"
    rows = torch.as_tensor(sample, device=DEV)
    check_records(codec.WindowStates(window.encoded, None, None,
                                     window.record_decay[rows], window.record_keys[rows],
                                     window.record_corrections[rows], window.positions[rows]),
                  [heads[int(i)] for i in sample], "after 18 tokens")


def test_full_window_is_left_untouched_and_reported():
    nheads = 4
    window = _qwen_boundary(nheads, False, seed=3)
    window.positions[:, 0] = wc.WINDOW
    inputs = wc.qwen_tokens(nheads, 1, seed=1)
    codec.device_error(DEV, clear=True)
    sentinel = torch.full((nheads, 128), 7.0, dtype=torch.bfloat16, device=DEV)
    before = window.record_keys.clone()
    codec.window_step_bf16(window, f32_dev(inputs["log_decay"][0]), bf16_dev(inputs["beta"][0]),
                           bf16_dev(inputs["keys"][0]), bf16_dev(inputs["queries"][0]),
                           bf16_dev(inputs["values"][0]), out=sentinel)
    torch.cuda.synchronize()
    assert bool((sentinel == 7.0).all())
    assert torch.equal(window.record_keys, before)
    assert (window.positions[:, 0] == wc.WINDOW).all()
    assert codec.device_error(DEV, clear=True) & codec.STATUS_WINDOW_FULL


def test_runtime_decode_matches_oracle():
    """The plugin runtime's step (runtime.py:750-845) for one slot over 18
    tokens: the window refit at token 16 and every bf16 output."""
    nheads, tokens = 32, 18
    experiment = GdnStateCodecExperiment(_native.library_dir(), "shadow", "quant_only", 0,
                                         "vector")
    rt = runtime_mod.GdnStateCodecRuntime(experiment, "model.layers.0.linear_attn")
    ssm = codec.synthesize_states(2, 1, nheads, layout="provider", seed=41,
                                  device=DEV).reshape(2, nheads, 128, 128)
    inputs = wc.qwen_tokens(nheads, tokens, seed=43)
    heads = None
    for t in range(tokens):
        def shaped(x, n):
            return x.reshape(1, 1, n, -1) if x.ndim == 2 else x.reshape(1, 1, n)
        out = rt.step(ssm, 1,
                      query=shaped(bf16_dev(inputs["queries"][t]), nheads // 2),
                      key=shaped(bf16_dev(inputs["keys"][t]), nheads // 2),
                      value=shaped(bf16_dev(inputs["values"][t]), nheads),
                      log_decay=shaped(f32_dev(inputs["log_decay"][t]), nheads),
                      beta=shaped(bf16_dev(inputs["beta"][t]), nheads),
                      query_scale=128 ** -0.5)
        torch.cuda.synchronize()
        slot = rt._slots[1]
        if heads is None:
            z, c, b = oracle.quantize(ssm[1].cpu().numpy(), "provider")
            heads = [oracle.WindowHead(z[i], c[i], b[i], layout="provider")
                     for i in range(nheads)]
        if t == wc.WINDOW:
            for h in heads:
                assert h.fold(0, round_storage=True) == 0
        pos = heads[0].position.value
        alpha = slot.record_decay[:, pos].cpu().numpy()
        want = [h.step(*oracle.qwen_token(alpha[i], inputs["beta"][t][i],
                                          inputs["keys"][t][i // 2], inputs["queries"][t][i // 2],
                                          inputs["values"][t][i]), round_storage=True)
                for i, h in enumerate(heads)]
        got = out.reshape(nheads, 128).view(torch.int16).cpu().numpy().view(np.uint16)
        assert np.array_equal(got, oracle.f32_to_bf16_array(np.stack(want))), f"token {t}"
    assert rt.boundary_refits == 1


@pytest.mark.parametrize("compensators, iterations, position",
                         [(False, 0, 7), (True, 0, 7), (True, 8, 7), (False, 0, 0), (True, 0, 0),
                          (False, 0, 16), (True, 0, 16)])
def test_refit_of_a_partial_window_matches_oracle(compensators, iterations, position):
    """A refit at position 7 (the probe case), of an empty window and of a
    full one: the folded boundary and the cleared window, bit-identical to the
    oracle.  20 heads, so the quant-only refit's CTAs each take more than one
    head through the staging pipeline."""
    case = wc.step_probe_case(states=20, position=position)
    window = window_from_case(case, "provider", compensators)
    heads = wc.window_heads(case, "provider", compensators)
    nxt = codec.window_refit(window, iterations)
    for h in heads:
        assert h.fold(iterations, round_storage=True) == 0
        if not compensators and iterations == 0:
            h.ck = h.cv = None
    _assert_boundary(nxt, heads, f"partial refit ({iterations})")
    check_records(nxt, heads, "partial refit")
    assert (nxt.compensator_keys is None) == (not compensators and iterations == 0)


def test_non_finite_refit_state_sets_the_status_bit():
    """A binary16 infinity in one head's record correction: the quant-only
    refit reports bit 4 (non-finite refit state) and not the fit's bit 2, the
    window is still cleared, and every other head's new boundary is still
    bit-identical to the oracle."""
    case = wc.step_probe_case(states=4, position=7)
    window = window_from_case(case, "provider", False)
    heads = wc.window_heads(case, "provider", False)
    window.record_corrections[2, 3, 17] = float("inf")
    codec.device_error(DEV, clear=True)
    nxt = codec.window_refit(window, 0)
    torch.cuda.synchronize()
    status = codec.device_error(DEV, clear=True)
    assert status & codec.STATUS_WINDOW_NON_FINITE
    assert not status & codec.STATUS_FIT_NON_FINITE
    for h in heads:
        assert h.fold(0, round_storage=True) == 0
        h.ck = h.cv = None
    keep = [0, 1, 3]
    sub = codec.WindowStates(
        codec.EncodedStates(nxt.encoded.codes[keep], nxt.encoded.smoothing[keep],
                            nxt.encoded.scales[keep], "provider"),
        None, None, nxt.record_decay[keep], nxt.record_keys[keep],
        nxt.record_corrections[keep], nxt.positions[keep])
    _assert_boundary(sub, [heads[i] for i in keep], "refit beside a non-finite head")
    assert bool((window.positions[:, 0] == 0).all())
    assert bool((window.record_corrections == 0).all())


def test_generic_step_sequence_matches_oracle():
    """16 generic (binary16) tokens from an empty window over a rank-4
    boundary, capsule layout: every output and record bit-identical to the
    oracle, the window full at the end."""
    nheads = 8
    states = codec.synthesize_states(1, 1, nheads, layout="capsule", seed=61,
                                     device=DEV).reshape(nheads, 128, 128)
    full = codec.full_encode(states, "capsule")
    window = codec.new_window(full.encoded, full.compensator_keys.half().contiguous(),
                              full.compensator_values.half().contiguous())
    heads = _oracle_heads_capsule(window)
    rng = np.random.default_rng(62)
    for t in range(wc.WINDOW):
        decay = (0.9 + 0.1 * rng.random(nheads)).astype(np.float32)
        vec = lambda s: wc.f16(rng.standard_normal((nheads, 128)) * s)  # noqa: E731
        key, read, query, value = vec(0.09), vec(0.09), vec(0.09), vec(1.0)
        out = codec.window_step(window, f32_dev(decay), f16_dev(key), f16_dev(read),
                                f16_dev(query), f16_dev(value))
        want = np.stack([h.step(decay[i], key[i], read[i], query[i], value[i])
                         for i, h in enumerate(heads)])
        assert np.array_equal(bits(out.cpu().numpy()), bits(want)), f"token {t}"
        check_records(window, heads, f"token {t}")
    assert bool((window.positions[:, 0] == wc.WINDOW).all())


def _oracle_heads_capsule(window):
    torch.cuda.synchronize()
    enc = window.encoded
    codes, c, b = enc.codes.cpu().numpy(), enc.smoothing.cpu().numpy(), enc.scales.cpu().numpy()
    ck = window.compensator_keys.float().cpu().numpy()
    cv = window.compensator_values.float().cpu().numpy()
    return [oracle.WindowHead(codes[i], c[i], b[i], ck[i], cv[i], layout="capsule")
            for i in range(codes.shape[0])]


def test_non_finite_token_sets_the_status_bit():
    nheads = 4
    window = _qwen_boundary(nheads, False, seed=71)
    inputs = wc.qwen_tokens(nheads, 1, seed=72)
    values = inputs["values"][0].copy()
    values[1, 5] = 0x7FC0  # bf16 NaN in head 1
    codec.device_error(DEV, clear=True)
    out = codec.window_step_bf16(window, f32_dev(inputs["log_decay"][0]),
                                 bf16_dev(inputs["beta"][0]), bf16_dev(inputs["keys"][0]),
                                 bf16_dev(inputs["queries"][0]), bf16_dev(values))
    torch.cuda.synchronize()
    bits = codec.device_error(DEV, clear=True)
    assert bits & codec.STATUS_WINDOW_NON_FINITE
    assert not bits & codec.STATUS_FIT_NON_FINITE  # the fit's bit stays its own
    assert torch.isnan(out[1].float()).any()
    assert torch.isfinite(out[0].float()).all() and torch.isfinite(out[2:].float()).all()
