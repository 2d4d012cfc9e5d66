# SPDX-License-Identifier: Apache-2.0
"""Torch-facing API of the B200 GDN state codec.

Every function validates its tensors, then enqueues one launch of the CUDA
library through the C ABI on the tensors' device and current CUDA stream.
Nothing here computes on the host; a non-zero status from the library raises
``RuntimeError`` (the reference runtime's behaviour, runtime.py:514-517).

Layouts (one head = one [128, 128] GDN recurrent-state matrix):
  ``"capsule"``  [key, value]  -- reference capsule order, [H, d_k, d_v]
  ``"provider"`` [value, key]  -- vLLM ssm_state order
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _native

KEY_DIMENSION = 128
VALUE_DIMENSION = 128
COMPENSATOR_RANK = 4
ELEMENTS = KEY_DIMENSION * VALUE_DIMENSION
LAYOUTS = {"capsule": 0, "provider": 1}
PAD_SLOT_ID = -1


@dataclass
class EncodedStates:
    """Quant-only encoded heads: int8 codes in the layout of the fp32 state
    they encode, smoothing per key and scales per value (17,408 B per head)."""

    codes: torch.Tensor
    smoothing: torch.Tensor
    scales: torch.Tensor
    layout: str = "capsule"

    @property
    def heads(self) -> int:
        return self.codes.numel() // ELEMENTS


def _ptr(tensor: torch.Tensor | None):
    return None if tensor is None else ctypes.c_void_p(tensor.data_ptr())


def _stream(device: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _check(tensor: torch.Tensor, name: str, dtype: torch.dtype, last: tuple[int, ...],
           device: torch.device | None = None) -> int:
    if not isinstance(tensor, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if tensor.device.type != "cuda":
        raise ValueError(f"{name} must be a CUDA tensor (got {tensor.device})")
    if device is not None and tensor.device != device:
        raise ValueError(f"{name} is on {tensor.device}, expected {device}")
    if tensor.dtype != dtype:
        raise ValueError(f"{name} must be {dtype} (got {tensor.dtype})")
    if not tensor.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    if last and (tensor.dim() < len(last) or tuple(tensor.shape[-len(last):]) != last):
        raise ValueError(f"{name} must end in shape {last} (got {tuple(tensor.shape)})")
    count = 1
    for size in tensor.shape[: tensor.dim() - len(last)]:
        count *= size
    return count


def _layout(layout: str) -> int:
    if layout not in LAYOUTS:
        raise ValueError(f"layout must be 'capsule' or 'provider' (got {layout!r})")
    return LAYOUTS[layout]


def _status(name: str, status: int) -> None:
    if status != 0:
        raise RuntimeError(f"GDN State Codec {name} launch failed: {status}")


def _heads_ok(heads: int) -> None:
    if heads < 1:
        raise ValueError("at least one state is required")
    if heads >= 2**32:
        raise ValueError("at most 2^32 - 1 states per launch")


def _compensators(encoded_heads: int, device, keys, values):
    if (keys is None) != (values is None):
        raise ValueError("compensator_keys and compensator_values go together")
    if keys is None:
        return None, None
    k = _check(keys, "compensator_keys", torch.float32, (KEY_DIMENSION, COMPENSATOR_RANK), device)
    v = _check(values, "compensator_values", torch.float32,
               (VALUE_DIMENSION, COMPENSATOR_RANK), device)
    if k != encoded_heads or v != encoded_heads:
        raise ValueError("compensators must have one [128, 4] block per state")
    return keys, values


def empty_encoded(heads_shape: tuple[int, ...], layout: str = "capsule",
                  device: torch.device | str = "cuda") -> EncodedStates:
    return EncodedStates(
        codes=torch.empty((*heads_shape, KEY_DIMENSION, VALUE_DIMENSION), dtype=torch.int8,
                          device=device),
        smoothing=torch.empty((*heads_shape, KEY_DIMENSION), dtype=torch.float32, device=device),
        scales=torch.empty((*heads_shape, VALUE_DIMENSION), dtype=torch.float32, device=device),
        layout=layout,
    )


def _check_encoded(encoded: EncodedStates, device=None) -> int:
    heads = _check(encoded.codes, "codes", torch.int8, (KEY_DIMENSION, VALUE_DIMENSION), device)
    dev = encoded.codes.device
    if _check(encoded.smoothing, "smoothing", torch.float32, (KEY_DIMENSION,), dev) != heads:
        raise ValueError("smoothing must have one [128] vector per state")
    if _check(encoded.scales, "scales", torch.float32, (VALUE_DIMENSION,), dev) != heads:
        raise ValueError("scales must have one [128] vector per state")
    _layout(encoded.layout)
    return heads


# ---------------------------------------------------------------------------
# Dense batches.

def quantize(states: torch.Tensor, layout: str = "capsule", *,
             out: EncodedStates | None = None) -> EncodedStates:
    """Fused smoothing + int8 quantize of every [128, 128] head in ``states``.

    Capsule layout calls ``initialize_launch_v3``; provider layout calls the
    plugin's ``provider_initialize_launch_v3``."""
    heads = _check(states, "states", torch.float32, (KEY_DIMENSION, VALUE_DIMENSION))
    _heads_ok(heads)
    code = _layout(layout)
    if out is None:
        out = empty_encoded(tuple(states.shape[:-2]), layout, states.device)
    if _check_encoded(out, states.device) != heads or out.layout != layout:
        raise ValueError("output buffers do not match the input states")
    name = ("statecentric_gdn_state_codec_provider_initialize_launch_v3" if code
            else "statecentric_gdn_state_codec_initialize_launch_v3")
    with torch.cuda.device(states.device):
        _status("quantize", _native.call(name, _stream(states.device), _ptr(states),
                                         _ptr(out.smoothing), _ptr(out.codes), _ptr(out.scales),
                                         heads))
    return out


def smoothing(states: torch.Tensor, layout: str = "provider",
              out: torch.Tensor | None = None) -> torch.Tensor:
    """Smoothing only.  Provider layout: ``provider_smoothing_launch_v2`` over
    all heads; capsule layout: ``smoothing_launch_v1`` once per head."""
    heads = _check(states, "states", torch.float32, (KEY_DIMENSION, VALUE_DIMENSION))
    _heads_ok(heads)
    code = _layout(layout)
    if out is None:
        out = torch.empty((*states.shape[:-2], KEY_DIMENSION), dtype=torch.float32,
                          device=states.device)
    if _check(out, "smoothing", torch.float32, (KEY_DIMENSION,), states.device) != heads:
        raise ValueError("smoothing output must have one [128] vector per state")
    with torch.cuda.device(states.device):
        stream = _stream(states.device)
        if code:
            _status("smoothing", _native.call(
                "statecentric_gdn_state_codec_provider_smoothing_launch_v2", stream,
                _ptr(states), _ptr(out), heads))
        else:
            flat_s, flat_o = states.view(-1, ELEMENTS), out.view(-1, KEY_DIMENSION)
            for h in range(heads):
                _status("smoothing", _native.call(
                    "statecentric_gdn_state_codec_smoothing_launch_v1", stream,
                    _ptr(flat_s[h]), _ptr(flat_o[h])))
    return out


def quantize_with_smoothing(states: torch.Tensor, smoothing_in: torch.Tensor,
                            layout: str = "provider", *,
                            out: EncodedStates | None = None) -> EncodedStates:
    """Quantize with the caller's smoothing.  Provider layout:
    ``provider_quantize_launch_v2``; capsule: ``quantize_launch_v1`` per head."""
    heads = _check(states, "states", torch.float32, (KEY_DIMENSION, VALUE_DIMENSION))
    _heads_ok(heads)
    code = _layout(layout)
    if _check(smoothing_in, "smoothing", torch.float32, (KEY_DIMENSION,), states.device) != heads:
        raise ValueError("smoothing must have one [128] vector per state")
    if out is None:
        out = empty_encoded(tuple(states.shape[:-2]), layout, states.device)
    _check_encoded(out, states.device)
    out.smoothing.copy_(smoothing_in)
    with torch.cuda.device(states.device):
        stream = _stream(states.device)
        if code:
            _status("quantize", _native.call(
                "statecentric_gdn_state_codec_provider_quantize_launch_v2", stream,
                _ptr(states), _ptr(smoothing_in), _ptr(out.codes), _ptr(out.scales), heads))
        else:
            fs, fc = states.view(-1, ELEMENTS), smoothing_in.view(-1, KEY_DIMENSION)
            fz, fb = out.codes.view(-1, ELEMENTS), out.scales.view(-1, VALUE_DIMENSION)
            for h in range(heads):
                _status("quantize", _native.call(
                    "statecentric_gdn_state_codec_quantize_launch_v1", stream,
                    _ptr(fs[h]), _ptr(fc[h]), _ptr(fz[h]), _ptr(fb[h])))
    return out


def dequantize(encoded: EncodedStates, *, compensator_keys: torch.Tensor | None = None,
               compensator_values: torch.Tensor | None = None,
               out: torch.Tensor | None = None) -> torch.Tensor:
    """fp32 reconstruction ((c * z) / 127) * b [+ K V^T], same layout as the codes."""
    heads = _check_encoded(encoded)
    _heads_ok(heads)
    device = encoded.codes.device
    ck, cv = _compensators(heads, device, compensator_keys, compensator_values)
    if out is None:
        out = torch.empty(encoded.codes.shape, dtype=torch.float32, device=device)
    if _check(out, "dense", torch.float32, (KEY_DIMENSION, VALUE_DIMENSION), device) != heads:
        raise ValueError("dense output must have one head per encoded head")
    name = ("statecentric_gdn_state_codec_provider_dequantize_launch_v2"
            if encoded.layout == "provider" else "statecentric_gdn_state_codec_dequantize_launch_v2")
    with torch.cuda.device(device):
        _status("dequantize", _native.call(
            name, _stream(device), _ptr(encoded.codes), _ptr(encoded.smoothing),
            _ptr(encoded.scales), _ptr(ck), _ptr(cv), _ptr(out), heads))
    return out


def encoded_projection(encoded: EncodedStates, queries: torch.Tensor, *,
                       compensator_keys: torch.Tensor | None = None,
                       compensator_values: torch.Tensor | None = None,
                       out: torch.Tensor | None = None) -> torch.Tensor:
    """o[h] = dequant(S_h)^T q_h from the int8 codes; q bf16 [..., 128] -> fp32."""
    heads = _check_encoded(encoded)
    _heads_ok(heads)
    device = encoded.codes.device
    if _check(queries, "queries", torch.bfloat16, (KEY_DIMENSION,), device) != heads:
        raise ValueError("queries must have one [128] bf16 vector per state")
    ck, cv = _compensators(heads, device, compensator_keys, compensator_values)
    if out is None:
        out = torch.empty(queries.shape, dtype=torch.float32, device=device)
    if _check(out, "outputs", torch.float32, (VALUE_DIMENSION,), device) != heads:
        raise ValueError("outputs must have one [128] vector per state")
    name = ("statecentric_gdn_state_codec_provider_encoded_projection_launch_v1"
            if encoded.layout == "provider"
            else "statecentric_gdn_state_codec_encoded_projection_launch_v1")
    with torch.cuda.device(device):
        _status("encoded projection", _native.call(
            name, _stream(device), _ptr(encoded.codes), _ptr(encoded.smoothing),
            _ptr(encoded.scales), _ptr(ck), _ptr(cv), _ptr(queries), _ptr(out), heads))
    return out


@dataclass
class FullEncoded:
    """The reference's full boundary of each head: int8 codes, smoothing and
    scales of the residual, the rank-4 compensators K [.., 128 keys, 4] and
    V [.., 128 values, 4], and the fp32 residual the codes encode."""

    encoded: EncodedStates
    compensator_keys: torch.Tensor
    compensator_values: torch.Tensor
    residual: torch.Tensor


def full_encode(states: torch.Tensor, layout: str = "capsule", *,
                status: torch.Tensor | None = None) -> FullEncoded:
    """FromDenseBoundary's encode (capsule.cpp:129-225) of every head: the
    rank-4 compensator fit, then smoothing + int8 quantize of the residual,
    bit-identical to the portable C++ codec.  Non-finite data sets
    STATUS_FIT_NON_FINITE (bit 2, value 4) of ``status`` (int32 device
    scalar, optional) and of the device error word."""
    heads = _check(states, "states", torch.float32, (KEY_DIMENSION, VALUE_DIMENSION))
    _heads_ok(heads)
    code = _layout(layout)
    device = states.device
    lead = tuple(states.shape[:-2])
    out = empty_encoded(lead, layout, device)
    keys = torch.empty((*lead, KEY_DIMENSION, COMPENSATOR_RANK), dtype=torch.float32, device=device)
    values = torch.empty((*lead, VALUE_DIMENSION, COMPENSATOR_RANK), dtype=torch.float32,
                         device=device)
    residual = torch.empty_like(states)
    with torch.cuda.device(device):
        _status("full encode", _native.call(
            "statecentric_gdn_state_codec_full_initialize_launch_v1", _stream(device), code,
            _ptr(states), _ptr(residual), _ptr(out.smoothing), _ptr(out.codes), _ptr(out.scales),
            _ptr(keys), _ptr(values), heads, _ptr(status)))
    return FullEncoded(out, keys, values, residual)


# ---------------------------------------------------------------------------
# The reference's capsule wire format (Serialize / Restore).

CAPSULE_BYTES = 21688
CAPSULE_STATUS = {
    0: "restored", 1: "capsule magic differs", 2: "checksum encoding is invalid",
    3: "checksum differs", 4: "quantization parameters differ",
    5: "identity or geometry differs", 6: "window position differs",
    7: "INT8 residual contains -128", 8: "boundary payload is invalid",
    9: "restored state is non-finite",
}


def _identity(geometry: str, generation: int, epoch: int):
    raw = geometry.encode("ascii")
    if len(raw) != 64 or any(c not in b"0123456789abcdef" for c in raw):
        raise ValueError("model geometry digest must be 64 lowercase hex characters")
    if generation <= 0 or epoch <= 0:
        raise ValueError("generation and epoch must be positive")
    return ctypes.c_char_p(raw), generation, epoch


def serialize_capsules(encoded: EncodedStates, *, geometry: str, generation: int, epoch: int,
                       compensator_keys: torch.Tensor | None = None,
                       compensator_values: torch.Tensor | None = None,
                       out: torch.Tensor | None = None) -> torch.Tensor:
    """The reference's Serialize of every encoded head: uint8 [heads, 21688],
    byte-identical to GdnStateCodecCapsule::Serialize (capsule.cpp:446-475)."""
    heads = _check_encoded(encoded)
    _heads_ok(heads)
    device = encoded.codes.device
    ck, cv = _compensators(heads, device, compensator_keys, compensator_values)
    geo, generation, epoch = _identity(geometry, generation, epoch)
    if out is None:
        out = torch.empty((heads, CAPSULE_BYTES), dtype=torch.uint8, device=device)
    if _check(out, "capsules", torch.uint8, (CAPSULE_BYTES,), device) != heads:
        raise ValueError("capsule buffer must hold one capsule per head")
    with torch.cuda.device(device):
        _status("capsule serialize", _native.call(
            "statecentric_gdn_state_codec_capsule_serialize_launch_v1", _stream(device),
            LAYOUTS[encoded.layout], _ptr(encoded.codes), _ptr(encoded.smoothing),
            _ptr(encoded.scales), _ptr(ck), _ptr(cv), geo, generation, epoch, _ptr(out), heads))
    return out


def restore_capsules(capsules: torch.Tensor, layout: str = "capsule", *, geometry: str,
                     generation: int, epoch: int):
    """The reference's Restore of each capsule, fail-closed per head: returns
    (EncodedStates, compensator_keys, compensator_values, status int32 [heads]);
    status 0 = restored, else the first failing check (CAPSULE_STATUS)."""
    heads = _check(capsules, "capsules", torch.uint8, (CAPSULE_BYTES,))
    _heads_ok(heads)
    device = capsules.device
    code = _layout(layout)
    geo, generation, epoch = _identity(geometry, generation, epoch)
    lead = tuple(capsules.shape[:-1])
    encoded = empty_encoded(lead, layout, device)
    keys = torch.zeros((*lead, KEY_DIMENSION, COMPENSATOR_RANK), dtype=torch.float32, device=device)
    values = torch.zeros((*lead, VALUE_DIMENSION, COMPENSATOR_RANK), dtype=torch.float32,
                         device=device)
    status = torch.empty(lead, dtype=torch.int32, device=device)
    with torch.cuda.device(device):
        _status("capsule restore", _native.call(
            "statecentric_gdn_state_codec_capsule_restore_launch_v1", _stream(device), code,
            _ptr(capsules), geo, generation, epoch, _ptr(encoded.codes), _ptr(encoded.smoothing),
            _ptr(encoded.scales), _ptr(keys), _ptr(values), _ptr(status), heads))
    return encoded, keys, values, status


def sha256_hex(data: bytes) -> str:
    """SHA-256 of host bytes by the library's own implementation (test support)."""
    buffer = ctypes.create_string_buffer(bytes(data), len(data)) if data else None
    out = ctypes.create_string_buffer(64)
    _status("sha256", _native.call("statecentric_gdn_state_codec_sha256_v1",
                                   ctypes.cast(buffer, ctypes.c_void_p) if buffer else None,
                                   len(data), out))
    return out.raw.decode("ascii")


# ---------------------------------------------------------------------------
# Slot-indexed caches ([num_slots, heads_per_slot, ...], slot-major).

def _slot_geometry(cache_heads: int, cache: torch.Tensor, slot_ids: torch.Tensor,
                   heads_per_slot: int) -> tuple[int, int]:
    if heads_per_slot < 1 or cache_heads % heads_per_slot:
        raise ValueError("cache head count must be a multiple of heads_per_slot")
    if (not isinstance(slot_ids, torch.Tensor) or slot_ids.dtype != torch.int32
            or slot_ids.dim() != 1 or not slot_ids.is_contiguous()
            or slot_ids.device != cache.device):
        raise ValueError("slot_ids must be a contiguous 1-D int32 tensor on the cache's device")
    count = slot_ids.numel()
    if count < 1:
        raise ValueError("at least one slot id is required")
    if cache_heads // heads_per_slot >= 2**31:
        raise ValueError("too many slots for int32 slot ids")
    return count, cache_heads // heads_per_slot


def quantize_indexed(state_cache: torch.Tensor, encoded_cache: EncodedStates,
                     slot_ids: torch.Tensor, heads_per_slot: int, *,
                     status: torch.Tensor | None = None) -> EncodedStates:
    """Encode the listed slots of ``state_cache`` into the same slots of
    ``encoded_cache``.  Ids of -1 are skipped; out-of-range ids are skipped and
    set bit 0 of ``status`` (int32 device scalar, optional)."""
    cache_heads = _check(state_cache, "state_cache", torch.float32,
                         (KEY_DIMENSION, VALUE_DIMENSION))
    device = state_cache.device
    if _check_encoded(encoded_cache, device) != cache_heads:
        raise ValueError("encoded cache must match the state cache")
    count, num_slots = _slot_geometry(cache_heads, state_cache, slot_ids, heads_per_slot)
    with torch.cuda.device(device):
        _status("indexed quantize", _native.call(
            "statecentric_gdn_state_codec_initialize_indexed_launch_v1", _stream(device),
            LAYOUTS[encoded_cache.layout], _ptr(state_cache), _ptr(encoded_cache.smoothing),
            _ptr(encoded_cache.codes), _ptr(encoded_cache.scales), _ptr(slot_ids), count,
            heads_per_slot, num_slots, _ptr(status)))
    return encoded_cache


def dequantize_indexed(encoded_cache: EncodedStates, state_cache: torch.Tensor,
                       slot_ids: torch.Tensor, heads_per_slot: int, *,
                       compensator_keys: torch.Tensor | None = None,
                       compensator_values: torch.Tensor | None = None,
                       status: torch.Tensor | None = None) -> torch.Tensor:
    cache_heads = _check_encoded(encoded_cache)
    device = encoded_cache.codes.device
    if _check(state_cache, "state_cache", torch.float32, (KEY_DIMENSION, VALUE_DIMENSION),
              device) != cache_heads:
        raise ValueError("state cache must match the encoded cache")
    ck, cv = _compensators(cache_heads, device, compensator_keys, compensator_values)
    count, num_slots = _slot_geometry(cache_heads, state_cache, slot_ids, heads_per_slot)
    with torch.cuda.device(device):
        _status("indexed dequantize", _native.call(
            "statecentric_gdn_state_codec_dequantize_indexed_launch_v1", _stream(device),
            LAYOUTS[encoded_cache.layout], _ptr(encoded_cache.codes),
            _ptr(encoded_cache.smoothing), _ptr(encoded_cache.scales), _ptr(ck), _ptr(cv),
            _ptr(state_cache), _ptr(slot_ids), count, heads_per_slot, num_slots, _ptr(status)))
    return state_cache


def encoded_projection_indexed(encoded_cache: EncodedStates, queries: torch.Tensor,
                               slot_ids: torch.Tensor, heads_per_slot: int, *,
                               compensator_keys: torch.Tensor | None = None,
                               compensator_values: torch.Tensor | None = None,
                               out: torch.Tensor | None = None,
                               status: torch.Tensor | None = None) -> torch.Tensor:
    """Projection gathered by slot: queries / outputs are compact
    [count, heads_per_slot, 128]; padded or invalid entries output zeros."""
    cache_heads = _check_encoded(encoded_cache)
    device = encoded_cache.codes.device
    ck, cv = _compensators(cache_heads, device, compensator_keys, compensator_values)
    count, num_slots = _slot_geometry(cache_heads, encoded_cache.codes, slot_ids, heads_per_slot)
    if _check(queries, "queries", torch.bfloat16, (KEY_DIMENSION,), device) != count * heads_per_slot:
        raise ValueError("queries must be [count, heads_per_slot, 128] bf16")
    if out is None:
        out = torch.empty(queries.shape, dtype=torch.float32, device=device)
    if _check(out, "outputs", torch.float32, (VALUE_DIMENSION,), device) != count * heads_per_slot:
        raise ValueError("outputs must be [count, heads_per_slot, 128] fp32")
    with torch.cuda.device(device):
        _status("indexed encoded projection", _native.call(
            "statecentric_gdn_state_codec_encoded_projection_indexed_launch_v1", _stream(device),
            LAYOUTS[encoded_cache.layout], _ptr(encoded_cache.codes),
            _ptr(encoded_cache.smoothing), _ptr(encoded_cache.scales), _ptr(ck), _ptr(cv),
            _ptr(queries), _ptr(out), _ptr(slot_ids), count, heads_per_slot, num_slots,
            _ptr(status)))
    return out


# ---------------------------------------------------------------------------
# Windowed decode (p = 16 records over the INT8 boundary).

WINDOW_SIZE = 16
POSITION_STRIDE = 8


@dataclass
class WindowStates:
    """Encoded heads with their decode windows (the window ABI's buffers):
    the INT8 boundary, binary16 rank-4 compensators (None: quant-only
    boundary), and per head up to 16 records {decay fp32, key fp16 [128],
    correction fp16 [128]} with the window position in ``positions[..., 0]``."""

    encoded: EncodedStates
    compensator_keys: torch.Tensor | None
    compensator_values: torch.Tensor | None
    record_decay: torch.Tensor
    record_keys: torch.Tensor
    record_corrections: torch.Tensor
    positions: torch.Tensor

    @property
    def heads(self) -> int:
        return self.encoded.heads


def new_window(encoded: EncodedStates, compensator_keys: torch.Tensor | None = None,
               compensator_values: torch.Tensor | None = None) -> WindowStates:
    """An empty window (position 0) over ``encoded``; compensators are
    binary16 [..., 128, 4] or None."""
    heads = _check_encoded(encoded)
    device = encoded.codes.device
    if (compensator_keys is None) != (compensator_values is None):
        raise ValueError("compensator_keys and compensator_values go together")
    if compensator_keys is not None:
        if (_check(compensator_keys, "compensator_keys", torch.float16,
                   (KEY_DIMENSION, COMPENSATOR_RANK), device) != heads or
                _check(compensator_values, "compensator_values", torch.float16,
                       (VALUE_DIMENSION, COMPENSATOR_RANK), device) != heads):
            raise ValueError("compensators must have one [128, 4] block per state")
    shape = tuple(encoded.codes.shape[:-2])
    return WindowStates(
        encoded, compensator_keys, compensator_values,
        record_decay=torch.zeros((*shape, WINDOW_SIZE), dtype=torch.float32, device=device),
        record_keys=torch.zeros((*shape, WINDOW_SIZE, KEY_DIMENSION), dtype=torch.float16,
                                device=device),
        record_corrections=torch.zeros((*shape, WINDOW_SIZE, VALUE_DIMENSION),
                                       dtype=torch.float16, device=device),
        positions=torch.zeros((*shape, POSITION_STRIDE), dtype=torch.int32, device=device))


def _check_window(window: WindowStates) -> int:
    heads = _check_encoded(window.encoded)
    dev = window.encoded.codes.device
    if window.compensator_keys is not None:
        if (_check(window.compensator_keys, "compensator_keys", torch.float16,
                   (KEY_DIMENSION, COMPENSATOR_RANK), dev) != heads or
                _check(window.compensator_values, "compensator_values", torch.float16,
                       (VALUE_DIMENSION, COMPENSATOR_RANK), dev) != heads):
            raise ValueError("compensators must have one [128, 4] block per state")
    for tensor, name, dtype, last in (
            (window.record_decay, "record_decay", torch.float32, (WINDOW_SIZE,)),
            (window.record_keys, "record_keys", torch.float16, (WINDOW_SIZE, KEY_DIMENSION)),
            (window.record_corrections, "record_corrections", torch.float16,
             (WINDOW_SIZE, VALUE_DIMENSION)),
            (window.positions, "positions", torch.int32, (POSITION_STRIDE,))):
        if _check(tensor, name, dtype, last, dev) != heads:
            raise ValueError(f"{name} must have one block per state")
    return heads


def _window_args(window: WindowStates):
    return (_ptr(window.encoded.codes), _ptr(window.encoded.smoothing),
            _ptr(window.encoded.scales), _ptr(window.compensator_keys),
            _ptr(window.compensator_values), _ptr(window.record_decay),
            _ptr(window.record_keys), _ptr(window.record_corrections), _ptr(window.positions))


def _window_launch(window: WindowStates):
    """(heads, pointer arguments) of a window's buffers, validated once per set
    of buffers: a later call with the same tensor objects at the same
    addresses, with the same dtype, shape and strides, reuses the result, so a
    decode loop pays for the checks of its per-token inputs only.  An in-place
    change of a buffer's metadata (resize_, transpose_, as_strided_, a new
    .data) changes that key and triggers a new check."""
    tensors = (window.encoded.codes, window.encoded.smoothing, window.encoded.scales,
               window.compensator_keys, window.compensator_values, window.record_decay,
               window.record_keys, window.record_corrections, window.positions)
    key = tuple(None if t is None else (t.data_ptr(), t.dtype, t.shape, t.stride())
                for t in tensors)
    cached = window.__dict__.get("_launch")
    if (cached is not None and cached[1] == key
            and all(a is b for a, b in zip(cached[0], tensors))):
        return cached[2], cached[3]
    heads = _check_window(window)
    launch = (heads, _window_args(window))
    window.__dict__["_launch"] = (tensors, key, *launch)
    return launch


def _vectors(heads: int, device, dtype, shapes: dict) -> None:
    for name, (tensor, count) in shapes.items():
        if _check(tensor, name, dtype, (KEY_DIMENSION,), device) != count:
            raise ValueError(f"{name} must be [{count}, 128] {dtype}")


def window_step_bf16(window: WindowStates, log_decay: torch.Tensor, beta: torch.Tensor,
                     keys: torch.Tensor, queries: torch.Tensor, values: torch.Tensor, *,
                     out: torch.Tensor | None = None) -> torch.Tensor:
    """One Qwen3.5 decode token for every head (ApplyToken, capsule.cpp:354-397):
    log_decay fp32 [H], beta bf16 [H], keys / queries bf16 [H/2, 128] (value
    heads 2j, 2j+1 share query/key head j), values bf16 [H, 128]; returns the
    bf16 outputs [H, 128] and appends one record per head.  The boundary must
    be provider layout.  Quant-only windows (no compensators) use the
    quant-only kernel."""
    heads, window_args = _window_launch(window)
    device = window.encoded.codes.device
    if window.encoded.layout != "provider":
        raise ValueError("the bf16 decode step reads provider-layout boundaries")
    if heads % 2:
        raise ValueError("the bf16 decode step needs an even number of heads")
    if _check(log_decay, "log_decay", torch.float32, (), device) != heads or \
            _check(beta, "beta", torch.bfloat16, (), device) != heads:
        raise ValueError("log_decay and beta must hold one value per head")
    _vectors(heads, device, torch.bfloat16, {"keys": (keys, heads // 2),
                                             "queries": (queries, heads // 2),
                                             "values": (values, heads)})
    if out is None:
        out = torch.empty((heads, VALUE_DIMENSION), dtype=torch.bfloat16, device=device)
    _vectors(heads, device, torch.bfloat16, {"outputs": (out, heads)})
    quant_only = window.compensator_keys is None
    name = ("windowed_gdn_step_bf16_quant_only_launch_v1" if quant_only
            else "windowed_gdn_step_bf16_launch_v1")
    with torch.cuda.device(device):
        _status("decode step", _native.call(
            "statecentric_gdn_state_codec_" + name, _stream(device), *window_args,
            _ptr(log_decay), _ptr(beta), _ptr(keys), _ptr(queries), _ptr(values), _ptr(out),
            heads))
    return out


def window_step(window: WindowStates, decay: torch.Tensor, write_keys: torch.Tensor,
                reads: torch.Tensor, queries: torch.Tensor, values: torch.Tensor, *,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """The generic decode step (windowed_gdn_step_launch_v1): decay fp32 [H]
    and fp16 [H, 128] write keys, reads, queries and values; fp32 outputs.
    The boundary must be capsule layout and carry compensators."""
    heads = _check_window(window)
    device = window.encoded.codes.device
    if window.encoded.layout != "capsule":
        raise ValueError("the generic decode step reads capsule-layout boundaries")
    if window.compensator_keys is None:
        raise ValueError("the generic decode step needs compensators")
    if _check(decay, "decay", torch.float32, (), device) != heads:
        raise ValueError("decay must hold one value per head")
    _vectors(heads, device, torch.float16, {"write_keys": (write_keys, heads),
                                            "reads": (reads, heads),
                                            "queries": (queries, heads),
                                            "values": (values, heads)})
    if out is None:
        out = torch.empty((heads, VALUE_DIMENSION), dtype=torch.float32, device=device)
    _vectors(heads, device, torch.float32, {"outputs": (out, heads)})
    with torch.cuda.device(device):
        _status("decode step", _native.call(
            "statecentric_gdn_state_codec_windowed_gdn_step_launch_v1", _stream(device),
            *_window_args(window), _ptr(decay), _ptr(write_keys), _ptr(reads), _ptr(queries),
            _ptr(values), _ptr(out), heads))
    return out


def window_refit(window: WindowStates, power_iterations: int = 0, *,
                 workspace: torch.Tensor | None = None) -> WindowStates:
    """Fold every head's window into a new boundary (DenseState then
    QuantizeBoundary with ``power_iterations`` sweeps per rank; 0 = quant-only
    boundary with zero compensators).  The records of ``window`` are cleared
    in place; the returned WindowStates holds the new boundary and shares the
    record buffers.  A quant-only window refit without power iterations stays
    quant-only (no compensators)."""
    heads = _check_window(window)
    device = window.encoded.codes.device
    if window.encoded.layout != "provider":
        raise ValueError("the boundary refit reads provider-layout boundaries")
    if not 0 <= power_iterations <= 32:
        raise ValueError("power_iterations must be in [0, 32]")
    shape = tuple(window.encoded.codes.shape[:-2])
    if workspace is None:
        workspace = torch.empty((*shape, VALUE_DIMENSION, KEY_DIMENSION), dtype=torch.float32,
                                device=device)
    if _check(workspace, "workspace", torch.float32, (VALUE_DIMENSION, KEY_DIMENSION),
              device) != heads:
        raise ValueError("workspace must hold one [128, 128] fp32 block per state")
    nxt = empty_encoded(shape, "provider", device)
    next_ck = torch.empty((*shape, KEY_DIMENSION, COMPENSATOR_RANK), dtype=torch.float16,
                          device=device)
    next_cv = torch.empty((*shape, VALUE_DIMENSION, COMPENSATOR_RANK), dtype=torch.float16,
                          device=device)
    with torch.cuda.device(device):
        _status("boundary refit", _native.call(
            "statecentric_gdn_state_codec_window_boundary_launch_v1", _stream(device),
            *_window_args(window), _ptr(nxt.codes), _ptr(nxt.smoothing), _ptr(nxt.scales),
            _ptr(next_ck), _ptr(next_cv), _ptr(workspace), heads, power_iterations))
    if window.compensator_keys is None and power_iterations == 0:
        next_ck = next_cv = None  # still a quant-only boundary (zero compensators)
    return WindowStates(nxt, next_ck, next_cv, window.record_decay, window.record_keys,
                        window.record_corrections, window.positions)


def dense_step(states: torch.Tensor, decay: torch.Tensor, keys: torch.Tensor,
               reads: torch.Tensor, queries: torch.Tensor, values: torch.Tensor, *,
               out: torch.Tensor | None = None) -> torch.Tensor:
    """fp32 GDN step in place on capsule-layout dense states
    (fp32_gdn_step_launch_v1): S = decay S + key (x) (value - S^T read);
    returns S^T query (fp32 [H, 128])."""
    heads = _check(states, "states", torch.float32, (KEY_DIMENSION, VALUE_DIMENSION))
    device = states.device
    if _check(decay, "decay", torch.float32, (), device) != heads:
        raise ValueError("decay must hold one value per head")
    _vectors(heads, device, torch.float16, {"keys": (keys, heads), "reads": (reads, heads),
                                            "queries": (queries, heads),
                                            "values": (values, heads)})
    if out is None:
        out = torch.empty((heads, VALUE_DIMENSION), dtype=torch.float32, device=device)
    _vectors(heads, device, torch.float32, {"outputs": (out, heads)})
    with torch.cuda.device(device):
        _status("dense step", _native.call(
            "statecentric_gdn_state_codec_fp32_gdn_step_launch_v1", _stream(device),
            _ptr(states), _ptr(decay), _ptr(keys), _ptr(reads), _ptr(queries), _ptr(values),
            _ptr(out), heads))
    return out


# ---------------------------------------------------------------------------
# Status and synthetic inputs.

# Bits of a caller's status word and of the sticky device error word.
STATUS_BAD_SLOT = 1             # bit 0: a slot id outside [-1, num_slots) was skipped
STATUS_WAIT_TIMEOUT = 2         # bit 1: a bounded device wait expired
STATUS_FIT_NON_FINITE = 4       # bit 2: a full-codec fit saw non-finite data
STATUS_WINDOW_FULL = 8          # bit 3: a decode step found a full window
STATUS_WINDOW_NON_FINITE = 16   # bit 4: a decode output or refit state was non-finite


def device_error(device: torch.device | str | int = "cuda", clear: bool = False) -> int:
    """Sticky error bits of the device (the STATUS_* values): 1 = invalid slot
    id, 2 = wait timeout, 4 = non-finite data in a full-codec fit, 8 = decode
    step on a full window, 16 = non-finite decode output or refit state."""
    bits = ctypes.c_uint32(0)
    with torch.cuda.device(device):
        _status("device error query", _native.call(
            "statecentric_gdn_state_codec_device_error_v1", ctypes.byref(bits), int(clear)))
    return int(bits.value)


def synthesize_states(slots: int, layers: int, heads_per_layer: int, *,
                      layout: str = "capsule", seed: int = 0, slot_base: int = 0,
                      device: torch.device | str = "cuda",
                      out: torch.Tensor | None = None) -> torch.Tensor:
    """Seeded GDN-like states [slots, layers, heads, 128, 128] generated on the
    device; slot ``slot_base + i`` is the same on any device and any shard."""
    code = _layout(layout)
    if out is None:
        out = torch.empty((slots, layers, heads_per_layer, KEY_DIMENSION, VALUE_DIMENSION),
                          dtype=torch.float32, device=device)
    heads = _check(out, "states", torch.float32, (KEY_DIMENSION, VALUE_DIMENSION))
    if heads != slots * layers * heads_per_layer:
        raise ValueError("output does not hold slots * layers * heads_per_layer heads")
    with torch.cuda.device(out.device):
        _status("synthesize states", _native.call(
            "statecentric_gdn_state_codec_synthesize_states_v1", _stream(out.device), _ptr(out),
            code, seed, slot_base, slots, layers, heads_per_layer))
    return out


def synthesize_queries(slots: int, layers: int, heads_per_layer: int, *, seed: int = 0,
                       slot_base: int = 0, device: torch.device | str = "cuda",
                       out: torch.Tensor | None = None) -> torch.Tensor:
    """Seeded bf16 queries [slots, layers, heads, 128], L2-normalised per head."""
    if out is None:
        out = torch.empty((slots, layers, heads_per_layer, KEY_DIMENSION), dtype=torch.bfloat16,
                          device=device)
    heads = _check(out, "queries", torch.bfloat16, (KEY_DIMENSION,))
    if heads != slots * layers * heads_per_layer:
        raise ValueError("output does not hold slots * layers * heads_per_layer queries")
    with torch.cuda.device(out.device):
        _status("synthesize queries", _native.call(
            "statecentric_gdn_state_codec_synthesize_queries_v1", _stream(out.device), _ptr(out),
            seed, slot_base, slots, layers, heads_per_layer))
    return out
