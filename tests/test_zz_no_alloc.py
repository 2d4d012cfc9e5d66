"""The full encode without a caller workspace (static device scratch).

Callers that cannot allocate device memory on the call path -- a serving
engine whose memory already belongs to its cache pools, or a host that owns
every device allocation -- call
statecentric_gdn_state_codec_full_initialize_static_launch_v1, which keeps the
residual between the fit and the int8 stage in a static device array of 64
heads instead of a workspace they would have to allocate.  This test calls it
through the C ABI twice in a row, with different inputs, and checks each call
against full_initialize_launch_v1 (the workspace entry point) bit for bit --
the same tolerance as every other parity test here.  It also checks that a
call above the array's 64-head limit is refused.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from gdn_state_codec import _native, codec

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
PREFIX = "statecentric_gdn_state_codec_"


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _static_encode(states: torch.Tensor, layout: int):
    heads = states.shape[0]
    smoothing = torch.empty((heads, 128), device=DEV)
    codes = torch.empty((heads, 128, 128), dtype=torch.int8, device=DEV)
    scales = torch.empty((heads, 128), device=DEV)
    keys = torch.empty((heads, 128, 4), device=DEV)
    values = torch.empty((heads, 128, 4), device=DEV)
    stream = ctypes.c_void_p(torch.cuda.current_stream(DEV).cuda_stream)
    status = _native.call(PREFIX + "full_initialize_static_launch_v1", stream, layout,
                          _ptr(states), _ptr(smoothing), _ptr(codes), _ptr(scales), _ptr(keys),
                          _ptr(values), heads, None)
    assert status == 0
    return codes, smoothing, scales, keys, values


def _bits_equal(a: torch.Tensor, b: torch.Tensor) -> bool:
    if a.dtype == torch.float32:
        return torch.equal(a.view(torch.int32), b.view(torch.int32))
    return torch.equal(a, b)


@pytest.mark.parametrize("layout", ["capsule", "provider"])
def test_static_scratch_full_encode_matches_workspace_entry_point(layout):
    code = 0 if layout == "capsule" else 1
    for call, heads in enumerate((40, 64)):  # two calls in a row, different inputs
        states = codec.synthesize_states(1, 1, heads, layout=layout, seed=100 + call,
                                         device=DEV).reshape(heads, 128, 128)
        got = _static_encode(states, code)
        want = codec.full_encode(states, layout)
        torch.cuda.synchronize()
        expected = (want.encoded.codes, want.encoded.smoothing, want.encoded.scales,
                    want.compensator_keys, want.compensator_values)
        for name, g, w in zip(("codes", "smoothing", "scales", "keys", "values"), got, expected):
            assert _bits_equal(g, w), f"call {call}: {name} differ"


def test_static_scratch_limit_is_enforced():
    states = torch.empty((65, 128, 128), device=DEV)
    out = torch.empty((65, 128, 128), device=DEV)
    stream = ctypes.c_void_p(torch.cuda.current_stream(DEV).cuda_stream)
    status = _native.call(PREFIX + "full_initialize_static_launch_v1", stream, 0, _ptr(states),
                          _ptr(out), _ptr(out), _ptr(out), _ptr(out), _ptr(out), 65, None)
    assert status == 1
