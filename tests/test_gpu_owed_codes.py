"""Exact codes owed across a launch.

An element whose scaled value lies next to a rounding boundary gets the
reference's exact code out of line. The quantizer does not write it with the
head. Each thread keeps up to two flagged heads and writes their exact codes
after the launch's last head. A thread that flags a third head patches it at
once from the head's shared arrays (gdn-state-codec_b200/csrc/quantize.cuh,
"owed exact codes").

These tests give every thread a flagged chunk in every head, in a launch of
about nine heads per block. So the kept entries, the late pass after the last
head and the immediate patches all run. The whole batch is compared bit for
bit with the oracle, fused and with caller-given smoothing, in both layouts.
The reference semantics are capsule.cpp:190-225.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from gdn_state_codec import codec

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _boundary_heads(count: int, seed: int) -> np.ndarray:
    """Heads whose elements sit next to rounding boundaries.

    Each row is a permutation of {1} and (n + 1/2) / 127, n = 0..126, with
    random signs. The rows form a Latin square, so every row has the same
    smoothing and every column has the maximum 1. Then the scaled value
    127 s / b of almost every element lies within the quantizer's ambiguity
    band of n + 1/2, and only the column maxima are left unflagged.
    """
    rng = np.random.default_rng(seed)
    base = np.concatenate([[1.0], (np.arange(127) + 0.5) / 127]).astype(np.float32)
    heads = np.empty((count, 128, 128), np.float32)
    for i in range(count):
        shift = int(rng.integers(0, 128))
        head = np.stack([np.roll(base, r + shift) for r in range(128)])
        heads[i] = head * np.where(rng.random((128, 128)) < 0.5, -1, 1).astype(np.float32)
    return heads


def _batch(layout: str, seed: int):
    sms = torch.cuda.get_device_properties(DEV).multi_processor_count
    count = 9 * 2 * sms + 5  # two quantize blocks per SM: about nine heads per block
    cap = _boundary_heads(count, seed)
    host = cap if layout == "capsule" else np.ascontiguousarray(cap.transpose(0, 2, 1))
    return host, torch.from_numpy(host).to(DEV)


def _bits(t: torch.Tensor) -> np.ndarray:
    a = t.cpu().numpy()
    return a.view(np.uint32) if a.dtype == np.float32 else a


@pytest.mark.parametrize("layout", ["capsule", "provider"])
def test_flagged_heads_in_every_block_fused(layout):
    host, states = _batch(layout, seed=41)
    enc = codec.quantize(states, layout)
    torch.cuda.synchronize()
    z, c, b = oracle.quantize(host, layout)
    got = _bits(enc.codes).reshape(z.shape)
    assert np.array_equal(got, z), f"{int((got != z).sum())} codes differ"
    assert np.array_equal(_bits(enc.smoothing).reshape(c.shape), c.view(np.uint32))
    assert np.array_equal(_bits(enc.scales).reshape(b.shape), b.view(np.uint32))


@pytest.mark.parametrize("layout", ["capsule", "provider"])
def test_flagged_heads_in_every_block_given_smoothing(layout):
    host, states = _batch(layout, seed=43)
    c = codec.smoothing(states, layout)
    staged = codec.quantize_with_smoothing(states, c, layout)
    torch.cuda.synchronize()
    z, c_ref, b = oracle.quantize(host, layout)
    assert np.array_equal(_bits(c).reshape(c_ref.shape), c_ref.view(np.uint32))
    got = _bits(staged.codes).reshape(z.shape)
    assert np.array_equal(got, z), f"{int((got != z).sum())} codes differ"
    assert np.array_equal(_bits(staged.scales).reshape(b.shape), b.view(np.uint32))
