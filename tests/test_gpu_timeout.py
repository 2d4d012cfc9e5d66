"""The bounded-wait failure path on the GPU, made to happen without a fault.

The quantizer, the capsule-code projection and the dense fp32 step stream
their inputs through shared memory with bulk copies completing on mbarriers,
and every wait on those barriers gives up after a limit (2 s in production),
reports bit 1 of the caller's status word and of the sticky device word, and
lets the kernel return.  The test-support launchers
(`quantize_wait_selftest_v1`, `encoded_projection_wait_selftest_v1`,
`fp32_gdn_step_wait_selftest_v1`) run the same kernels with the barriers
armed for a copy that is never issued, so each wait runs out (a flag that
nothing sets) after a 1 ms limit with nothing in flight.  The test checks the
status bits, that the context still works, and that the next ordinary launch
is bit-exact against the oracle.  No GPU is faulted, trapped or hung.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

import oracle
from gdn_state_codec import _native, codec

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")
LIMIT_NS = 1_000_000  # 1 ms
TIMEOUT_BIT = 2


def ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def stream():
    return ctypes.c_void_p(torch.cuda.current_stream(DEV).cuda_stream)


def check_quantize_exact(states, encoded):
    z, c, b = oracle.quantize(states.cpu().numpy().reshape(-1, 128, 128), "capsule")
    assert np.array_equal(encoded.codes.cpu().numpy().reshape(-1, 128, 128), z)
    assert np.array_equal(encoded.smoothing.cpu().numpy().reshape(-1, 128).view(np.uint32),
                          c.view(np.uint32))
    assert np.array_equal(encoded.scales.cpu().numpy().reshape(-1, 128).view(np.uint32),
                          b.view(np.uint32))
    return z, c, b


@pytest.mark.parametrize("heads", [4, 600])
def test_quantize_wait_runs_out_and_reports(heads):
    codec.device_error(DEV, clear=True)
    states = codec.synthesize_states(1, 1, heads, device=DEV, seed=11)
    enc = codec.empty_encoded((1, 1, heads), "capsule", DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    rc = _native.call("statecentric_gdn_state_codec_quantize_wait_selftest_v1", stream(),
                      ptr(states), ptr(enc.smoothing), ptr(enc.codes), ptr(enc.scales), heads,
                      LIMIT_NS, ptr(status))
    assert rc == 0
    torch.cuda.synchronize(DEV)  # the kernel returned: the context is usable
    assert int(status.item()) & TIMEOUT_BIT
    assert codec.device_error(DEV, clear=True) & TIMEOUT_BIT
    # The next ordinary launch over the same buffers is exact and reports nothing.
    codec.quantize(states, out=enc)
    torch.cuda.synchronize(DEV)
    check_quantize_exact(states, enc)
    assert codec.device_error(DEV) & TIMEOUT_BIT == 0


@pytest.mark.parametrize("heads", [4, 600])
def test_projection_wait_runs_out_and_reports(heads):
    codec.device_error(DEV, clear=True)
    states = codec.synthesize_states(1, 1, heads, device=DEV, seed=12)
    queries = codec.synthesize_queries(1, 1, heads, device=DEV, seed=12)
    enc = codec.quantize(states)
    out = torch.empty((1, 1, heads, 128), dtype=torch.float32, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    rc = _native.call("statecentric_gdn_state_codec_encoded_projection_wait_selftest_v1",
                      stream(), ptr(enc.codes), ptr(enc.smoothing), ptr(enc.scales),
                      ptr(queries), ptr(out), heads, LIMIT_NS, ptr(status))
    assert rc == 0
    torch.cuda.synchronize(DEV)
    assert int(status.item()) & TIMEOUT_BIT
    assert codec.device_error(DEV, clear=True) & TIMEOUT_BIT
    codec.encoded_projection(enc, queries, out=out)
    torch.cuda.synchronize(DEV)
    z, c, b = check_quantize_exact(states, enc)
    want = oracle.project(z, c, b, queries.float().cpu().numpy().reshape(-1, 128))
    assert np.array_equal(out.cpu().numpy().reshape(-1, 128), want)
    assert codec.device_error(DEV) & TIMEOUT_BIT == 0


@pytest.mark.parametrize("heads", [4, 600])
def test_dense_step_wait_runs_out_and_reports(heads):
    """The dense fp32 step (fp32_gdn_step_launch_v1) on the same failure
    path: the wait on its first landing buffer runs out, bit 1 of the sticky
    word is set, and no state or output is written."""
    codec.device_error(DEV, clear=True)
    states = codec.synthesize_states(1, 1, heads, device=DEV, seed=13).reshape(heads, 128, 128)
    before = states.clone()
    gen = torch.Generator(device=DEV).manual_seed(5)
    decay = 0.9 + 0.1 * torch.rand(heads, generator=gen, device=DEV)

    def vectors():
        return (torch.randn((heads, 128), generator=gen, device=DEV) / 11.3).half()

    keys, reads, queries, values = vectors(), vectors(), vectors(), vectors()
    out = torch.full((heads, 128), 7.0, device=DEV)
    rc = _native.call("statecentric_gdn_state_codec_fp32_gdn_step_wait_selftest_v1", stream(),
                      ptr(states), ptr(decay), ptr(keys), ptr(reads), ptr(queries), ptr(values),
                      ptr(out), heads, LIMIT_NS)
    assert rc == 0
    torch.cuda.synchronize(DEV)
    assert codec.device_error(DEV, clear=True) & TIMEOUT_BIT
    assert torch.equal(states.view(torch.int32), before.view(torch.int32))
    assert bool((out == 7.0).all())
    # The next ordinary step is exact against the oracle and reports nothing.
    got = codec.dense_step(states, decay, keys, reads, queries, values)
    torch.cuda.synchronize(DEV)
    host = before.cpu().numpy().copy()
    f32 = lambda t: t.float().cpu().numpy()  # noqa: E731
    d, k, r, q, v = decay.cpu().numpy(), f32(keys), f32(reads), f32(queries), f32(values)
    want = np.stack([oracle.dense_step(host[i], d[i], k[i], r[i], q[i], v[i])
                     for i in range(heads)])
    assert np.array_equal(got.cpu().numpy().view(np.uint32), want.view(np.uint32))
    assert np.array_equal(states.cpu().numpy().view(np.uint32), host.view(np.uint32))
    assert codec.device_error(DEV) & TIMEOUT_BIT == 0
