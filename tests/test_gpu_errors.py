"""GPU-side error behaviour of the C ABI: rejected arguments return 1 before
any launch (gdn_state_codec_kernel.h conventions, mirroring the reference's
launchers, e.g. native/ascendc/gdn_state_codec/kernel/gdn_state_codec_
smoothing.cpp:144-146), loader-compatibility entry points return 5, and the
context stays usable afterwards."""

from __future__ import annotations

import ctypes

import pytest
import torch

from gdn_state_codec import _native, codec

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")


def p(t):
    return ctypes.c_void_p(t.data_ptr())


def test_rejections_then_success():
    states = codec.synthesize_states(1, 1, 4, device=DEV)
    enc = codec.empty_encoded((1, 1, 4), "provider", DEV)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    name = "statecentric_gdn_state_codec_provider_initialize_launch_v3"
    assert _native.call(name, stream, None, p(enc.smoothing), p(enc.codes), p(enc.scales), 4) == 1
    assert _native.call(name, stream, p(states), p(enc.smoothing), p(enc.codes), p(enc.scales), 0) == 1
    misaligned = ctypes.c_void_p(states.data_ptr() + 4)
    assert _native.call(name, stream, misaligned, p(enc.smoothing), p(enc.codes),
                        p(enc.scales), 1) == 1
    # one compensator without the other
    assert _native.call("statecentric_gdn_state_codec_dequantize_launch_v2", stream,
                        p(enc.codes), p(enc.smoothing), p(enc.scales), p(states), None,
                        p(states), 4) == 1
    # bad layout flag on an indexed entry point
    ids = torch.zeros(1, dtype=torch.int32, device=DEV)
    assert _native.call("statecentric_gdn_state_codec_initialize_indexed_launch_v1", stream, 2,
                        p(states), p(enc.smoothing), p(enc.codes), p(enc.scales), p(ids), 1, 4, 1,
                        None) == 1
    assert _native.call("statecentric_gdn_state_codec_windowed_gdn_step_launch_v1",
                        *([None] * 16), 1) == 1
    assert _native.call("statecentric_gdn_state_codec_window_boundary_launch_v1",
                        *([None] * 16), 1, 0) == 1
    # A valid launch still works afterwards and the device reports no error.
    assert _native.call(name, stream, p(states), p(enc.smoothing), p(enc.codes), p(enc.scales), 4) == 0
    torch.cuda.synchronize()
    assert codec.device_error(DEV) & 2 == 0


def test_python_api_validation():
    states = codec.synthesize_states(1, 1, 2, device=DEV)
    with pytest.raises(ValueError):
        codec.quantize(states.cpu())
    with pytest.raises(ValueError):
        codec.quantize(states.double())
    with pytest.raises(ValueError):
        codec.quantize(states.transpose(-1, -2))
    with pytest.raises(ValueError):
        codec.quantize(states, layout="columns")
    enc = codec.quantize(states)
    with pytest.raises(ValueError):
        codec.encoded_projection(enc, torch.zeros(2, 128, device=DEV))  # fp32 query


def test_window_api_validation():
    """The window API refuses what its kernels cannot take, before any launch."""
    codec.device_error(DEV, clear=True)
    states = codec.synthesize_states(1, 1, 4, layout="provider", device=DEV).reshape(4, 128, 128)
    enc = codec.quantize(states, "provider")
    window = codec.new_window(enc)
    bf = torch.bfloat16
    token = dict(log_decay=torch.zeros(4, device=DEV), beta=torch.zeros(4, dtype=bf, device=DEV),
                 keys=torch.zeros(2, 128, dtype=bf, device=DEV),
                 queries=torch.zeros(2, 128, dtype=bf, device=DEV),
                 values=torch.zeros(4, 128, dtype=bf, device=DEV))
    codec.window_step_bf16(window, **token)  # valid
    torch.cuda.synchronize()
    with pytest.raises(ValueError, match="one value per head"):
        codec.window_step_bf16(window, **{**token, "log_decay": torch.zeros(3, device=DEV)})
    with pytest.raises(ValueError):
        codec.window_step_bf16(window, **{**token, "keys": torch.zeros(4, 128, dtype=bf, device=DEV)})
    with pytest.raises(ValueError):
        codec.window_step_bf16(window, **{**token, "values": token["values"].float()})
    odd = codec.new_window(codec.quantize(states[:3].contiguous(), "provider"))
    with pytest.raises(ValueError, match="even number of heads"):
        codec.window_step_bf16(odd, **token)
    capsule = codec.new_window(codec.quantize(states, "capsule"))
    with pytest.raises(ValueError, match="provider-layout"):
        codec.window_step_bf16(capsule, **token)
    with pytest.raises(ValueError, match="needs compensators"):
        codec.window_step(capsule, torch.ones(4, device=DEV),
                          *[torch.zeros(4, 128, dtype=torch.float16, device=DEV)] * 4)
    with pytest.raises(ValueError, match="power_iterations"):
        codec.window_refit(window, 33)
    with pytest.raises(ValueError, match="provider-layout"):
        codec.window_refit(capsule, 0)
    with pytest.raises(ValueError, match="go together"):
        codec.new_window(enc, torch.zeros(4, 128, 4, dtype=torch.float16, device=DEV), None)
    with pytest.raises(ValueError):
        codec.new_window(enc, torch.zeros(4, 128, 4, device=DEV),
                         torch.zeros(4, 128, 4, device=DEV))  # fp32, not binary16
    # nothing above reached the device with bad arguments
    assert codec.device_error(DEV) & ~codec.STATUS_WINDOW_FULL == 0
