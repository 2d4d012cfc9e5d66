"""CPU tests of the torch-facing API's argument checks (gdn_state_codec.codec).

Every check runs before any CUDA call, so host tensors, wrong dtypes and
wrong shapes are refused here without a GPU: the API fails loudly instead of
falling back to anything on the host.
"""

from __future__ import annotations

import pytest
import torch

from gdn_state_codec import codec


def test_host_tensors_are_refused():
    states = torch.zeros((2, 128, 128), dtype=torch.float32)
    with pytest.raises(ValueError, match="must be a CUDA tensor"):
        codec.quantize(states, "capsule")
    with pytest.raises(ValueError, match="must be a CUDA tensor"):
        codec.full_encode(states, "provider")
    with pytest.raises(ValueError, match="must be a CUDA tensor"):
        codec.smoothing(states, "provider")


def test_non_tensors_are_refused():
    with pytest.raises(TypeError, match="must be a torch.Tensor"):
        codec.quantize([[0.0] * 128] * 128, "capsule")


def test_unknown_layout_is_refused():
    with pytest.raises(ValueError, match="layout must be"):
        codec._layout("transposed")


def test_capsule_identity_rules():
    good = "0123456789abcdef" * 4
    codec._identity(good, 1, 1)
    with pytest.raises(ValueError, match="64 lowercase hex"):
        codec._identity(good.upper(), 1, 1)
    with pytest.raises(ValueError, match="64 lowercase hex"):
        codec._identity(good[:-1], 1, 1)
    with pytest.raises(ValueError, match="positive"):
        codec._identity(good, 0, 1)
    with pytest.raises(ValueError, match="positive"):
        codec._identity(good, 1, 0)


def test_capsule_status_names_cover_restore_checks():
    # Restore's checks in the reference's order (capsule.cpp:477-578), 0 = restored.
    assert sorted(codec.CAPSULE_STATUS) == list(range(10))
    assert codec.CAPSULE_BYTES == 21688


def test_window_buffers_are_validated_once_per_set_of_buffers(monkeypatch):
    calls = []
    monkeypatch.setattr(codec, "_check_window", lambda w: calls.append("check") or 4)
    monkeypatch.setattr(codec, "_window_args", lambda w: ("args",))

    def tensor(*shape, dtype=torch.float32):
        return torch.zeros(shape, dtype=dtype)

    window = codec.WindowStates(
        codec.EncodedStates(tensor(4, 128, 128, dtype=torch.int8), tensor(4, 128),
                            tensor(4, 128), "provider"),
        None, None, tensor(4, 16), tensor(4, 16, 128, dtype=torch.float16),
        tensor(4, 16, 128, dtype=torch.float16), tensor(4, 8, dtype=torch.int32))
    assert codec._window_launch(window) == (4, ("args",))
    assert codec._window_launch(window) == (4, ("args",))
    assert calls == ["check"]
    window.positions = tensor(4, 8, dtype=torch.int32)  # a new buffer: checked again
    codec._window_launch(window)
    assert calls == ["check", "check"]
    # In-place metadata changes keep the object and the address but change
    # the shape or strides: each one is checked again.
    window.record_decay.resize_(2, 16)  # smaller: same storage, same address
    codec._window_launch(window)
    assert calls == ["check"] * 3
    window.encoded.smoothing.t_()
    codec._window_launch(window)
    assert calls == ["check"] * 4
    window.encoded.scales.as_strided_((4, 64), (128, 1))
    codec._window_launch(window)
    assert calls == ["check"] * 5
    codec._window_launch(window)  # unchanged since: cached
    assert calls == ["check"] * 5
    assert window == codec.WindowStates(window.encoded, None, None, window.record_decay,
                                        window.record_keys, window.record_corrections,
                                        window.positions)  # the cache is not a field
