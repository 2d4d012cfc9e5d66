"""CPU tests of the capsule wire-format support: the library's SHA-256
(FIPS 180-4, constants derived from their definition, the same code the
capsule kernels run on the device) against hashlib and the standard's
examples, and the argument checks of the serialize / restore entry points."""

from __future__ import annotations

import hashlib
import os

import pytest

from gdn_state_codec import _native, codec

PREFIX = "statecentric_gdn_state_codec_"
ALIGNED = 0x10000
GEOMETRY = b"a" * 64


@pytest.mark.parametrize("size", [0, 1, 3, 55, 56, 57, 63, 64, 65, 119, 120, 127, 128, 1000,
                                  21624, 100003])
def test_sha256_matches_hashlib(size):
    data = os.urandom(size)
    assert codec.sha256_hex(data) == hashlib.sha256(data).hexdigest()


def test_sha256_standard_examples():
    # FIPS 180-4 example messages (one block, two blocks, empty).
    assert codec.sha256_hex(b"abc") == (
        "ba7816bf8f01cfea414140de5dae2223b00361a396177a9cb410ff61f20015ad")
    assert codec.sha256_hex(b"abcdbcdecdefdefgefghfghighijhijkijkljklmklmnlmnomnopnopq") == (
        "248d6a61d20638b8e5c026930c3e6039a33ce45964ff2167f6ecedd419db06c1")
    assert codec.sha256_hex(b"") == (
        "e3b0c44298fc1c149afbf4c8996fb92427ae41e4649b934ca495991b7852b855")


def test_capsule_entry_points_validate_identity_and_buffers():
    a, n = ALIGNED, None
    serialize = PREFIX + "capsule_serialize_launch_v1"
    restore = PREFIX + "capsule_restore_launch_v1"
    ok = (n, 0, a, a, a, n, n, GEOMETRY, 7, 11, a, 1)
    bad_args = [
        (n, 2, a, a, a, n, n, GEOMETRY, 7, 11, a, 1),           # layout
        (n, 0, a, a, a, n, n, b"A" * 64, 7, 11, a, 1),          # uppercase digest
        (n, 0, a, a, a, n, n, b"a" * 63 + b"g", 7, 11, a, 1),   # not hex
        (n, 0, a, a, a, n, n, GEOMETRY, 0, 11, a, 1),           # generation 0
        (n, 0, a, a, a, n, n, GEOMETRY, 7, 0, a, 1),            # epoch 0
        (n, 0, a, a, a, a, n, GEOMETRY, 7, 11, a, 1),           # lone compensator
        (n, 0, a, a, a, n, n, GEOMETRY, 7, 11, a + 4, 1),       # capsules not 8-byte aligned
        (n, 0, a, a, a, n, n, GEOMETRY, 7, 11, a, 0),           # no states
        (n, 0, a, a, a, n, n, None, 7, 11, a, 1),               # no identity
    ]
    for args in bad_args:
        assert _native.call(serialize, *args) == 1, args
    assert ok  # the valid argument list differs from each rejected one in one place
    assert _native.call(restore, n, 0, a, b"A" * 64, 7, 11, a, a, a, a, a, a, 1) == 1
    assert _native.call(restore, n, 0, a, GEOMETRY, 7, 11, a, a, a, a, a, n, 1) == 1
    assert _native.call(restore, n, 0, a + 4, GEOMETRY, 7, 11, a, a, a, a, a, a, 1) == 1


def test_python_identity_checks():
    with pytest.raises(ValueError, match="64 lowercase hex"):
        codec._identity("abc", 1, 1)
    with pytest.raises(ValueError, match="positive"):
        codec._identity("a" * 64, 0, 1)
