"""GPU tests of the capsule wire format against the reference library's own
Serialize / Restore (native/src, compiled into oracle/_ref): byte-identical
capsules, round trips, and the same fail-closed verdict on corrupted ones."""

from __future__ import annotations

import hashlib
import struct

import numpy as np
import pytest
import torch

import oracle
from gdn_state_codec import codec

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not oracle.ref_available(), reason="reference library not built")]
DEV = torch.device("cuda:0")
GEOMETRY = "0123456789abcdef" * 4
GENERATION, EPOCH = 3, 42
HEADER, ELEMENTS = 120, 128 * 128


def dense_heads(n: int = 6) -> np.ndarray:
    rng = np.random.default_rng(21)
    heads = []
    for _ in range(n - 2):
        h = (rng.standard_normal((128, 128)) * 10.0 ** (-3.0 * rng.random())).astype(np.float32)
        h[rng.random((128, 128)) < 0.01] = 0.0
        heads.append(h)
    heads.append(np.zeros((128, 128), np.float32))
    holes = (rng.standard_normal((128, 128))).astype(np.float32)
    holes[:, 3] = 0.0
    heads.append(holes)
    return np.stack(heads)


def parse(capsule: bytes):
    """Planes of a serialized boundary capsule."""
    codes = np.frombuffer(capsule, np.int8, ELEMENTS, HEADER).reshape(128, 128)
    floats = np.frombuffer(capsule, "<f4", 256 + 1024, HEADER + ELEMENTS)
    return codes, floats[:128], floats[128:256], floats[256:768].reshape(128, 4), \
        floats[768:].reshape(128, 4)


def reference_capsules(dense: np.ndarray) -> list[bytes]:
    return [oracle.ref_serialize_head(d, GEOMETRY, GENERATION, EPOCH) for d in dense]


@pytest.fixture(scope="module")
def capsules():
    dense = dense_heads()
    return dense, reference_capsules(dense)


@pytest.mark.parametrize("layout", ["capsule", "provider"])
def test_serialize_is_byte_identical_to_reference(capsules, layout):
    _, ref = capsules
    planes = [parse(c) for c in ref]
    codes = np.stack([p[0] for p in planes])
    if layout == "provider":
        codes = np.ascontiguousarray(codes.transpose(0, 2, 1))
    enc = codec.EncodedStates(torch.from_numpy(codes).to(DEV),
                              torch.from_numpy(np.stack([p[1] for p in planes])).to(DEV),
                              torch.from_numpy(np.stack([p[2] for p in planes])).to(DEV), layout)
    ck = torch.from_numpy(np.stack([p[3] for p in planes])).to(DEV)
    cv = torch.from_numpy(np.stack([p[4] for p in planes])).to(DEV)
    out = codec.serialize_capsules(enc, geometry=GEOMETRY, generation=GENERATION, epoch=EPOCH,
                                   compensator_keys=ck, compensator_values=cv)
    got = out.cpu().numpy()
    for i, c in enumerate(ref):
        assert got[i].tobytes() == c, f"capsule {i} differs"


def test_gpu_full_encode_then_serialize_equals_reference_serialize(capsules):
    dense, ref = capsules
    full = codec.full_encode(torch.from_numpy(dense).to(DEV), "capsule")
    out = codec.serialize_capsules(full.encoded, geometry=GEOMETRY, generation=GENERATION,
                                   epoch=EPOCH, compensator_keys=full.compensator_keys,
                                   compensator_values=full.compensator_values)
    got = out.cpu().numpy()
    for i, c in enumerate(ref):
        assert got[i].tobytes() == c, f"head {i}: GPU full encode + serialize differs"


@pytest.mark.parametrize("layout", ["capsule", "provider"])
def test_restore_round_trip(capsules, layout):
    _, ref = capsules
    blob = torch.from_numpy(np.frombuffer(b"".join(ref), np.uint8).reshape(len(ref), -1).copy())
    enc, ck, cv, status = codec.restore_capsules(blob.to(DEV), layout, geometry=GEOMETRY,
                                                 generation=GENERATION, epoch=EPOCH)
    torch.cuda.synchronize()
    assert status.cpu().tolist() == [0] * len(ref)
    for i, c in enumerate(ref):
        codes, sm, sc, k, v = parse(c)
        got_codes = enc.codes[i].cpu().numpy()
        assert np.array_equal(got_codes if layout == "capsule" else got_codes.T, codes)
        for got, want in ((enc.smoothing[i], sm), (enc.scales[i], sc), (ck[i], k), (cv[i], v)):
            assert np.array_equal(got.cpu().numpy().view(np.uint32), want.view(np.uint32))
        assert oracle.ref_restore_capsule(c, GEOMETRY, GENERATION, EPOCH)[0]


def _rehash(buf: bytearray) -> bytearray:
    buf[-64:] = hashlib.sha256(bytes(buf[:-64])).hexdigest().encode()
    return buf


def _set_f32(buf: bytearray, offset: int, value: float) -> None:
    buf[offset:offset + 4] = struct.pack("<f", value)


def _corruptions(c: bytes):
    smoothing = HEADER + ELEMENTS
    scales = smoothing + 512
    keys = scales + 512
    cases = []
    b = bytearray(c); b[0] = ord("X"); cases.append(("magic", b, 1, "magic differs"))
    b = bytearray(c); b[-64:] = bytes(c[-64:]).upper()
    cases.append(("digest case", b, 2, "checksum encoding is invalid"))
    b = bytearray(c); b[HEADER + 77] ^= 0x01; cases.append(("payload flip", b, 3, "checksum differs"))
    b = bytearray(c); b[12:16] = struct.pack("<I", 8)
    cases.append(("window size", _rehash(b), 4, "quantization parameters differ"))
    b = bytearray(c); b[36:44] = struct.pack("<Q", EPOCH + 1)
    cases.append(("epoch", _rehash(b), 5, "identity or geometry differs"))
    b = bytearray(c); b[52:56] = struct.pack("<I", 1)
    cases.append(("window phase", _rehash(b), 6, "window phase differs"))
    b = bytearray(c); b[HEADER + 5] = 0x80
    cases.append(("code -128", _rehash(b), 7, "contains -128"))
    b = bytearray(c); _set_f32(b, smoothing + 12, 0.0)
    cases.append(("smoothing 0", _rehash(b), 8, "boundary payload is invalid"))
    b = bytearray(c); _set_f32(b, scales + 28, float("nan"))
    cases.append(("scale nan", _rehash(b), 8, "boundary payload is invalid"))
    b = bytearray(c); _set_f32(b, keys + 40, float("inf"))
    cases.append(("key inf", _rehash(b), 8, "boundary payload is invalid"))
    b = bytearray(c); b[HEADER] = 127; _set_f32(b, smoothing, 3e38); _set_f32(b, scales, 3e38)
    cases.append(("dense overflow", _rehash(b), 9, "restored state is non-finite"))
    return cases


def test_restore_rejects_exactly_where_the_reference_rejects(capsules):
    _, ref = capsules
    cases = _corruptions(ref[0])
    blob = torch.from_numpy(np.frombuffer(b"".join(bytes(b) for _, b, _, _ in cases),
                                          np.uint8).reshape(len(cases), -1).copy()).to(DEV)
    _, _, _, status = codec.restore_capsules(blob, "capsule", geometry=GEOMETRY,
                                             generation=GENERATION, epoch=EPOCH)
    got = status.cpu().tolist()
    for (name, data, expected, message), code in zip(cases, got):
        assert code == expected, f"{name}: status {code}, expected {expected}"
        accepted, reason = oracle.ref_restore_capsule(bytes(data), GEOMETRY, GENERATION, EPOCH)
        assert not accepted and message in reason, f"{name}: reference said {reason!r}"
    # a wrong expected identity rejects every head
    good = torch.from_numpy(np.frombuffer(ref[1], np.uint8).copy()).reshape(1, -1).to(DEV)
    _, _, _, status = codec.restore_capsules(good, "capsule", geometry="f" * 64,
                                             generation=GENERATION, epoch=EPOCH)
    assert status.item() == 5
