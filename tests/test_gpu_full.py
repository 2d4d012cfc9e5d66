"""GPU parity of the full codec (rank-4 compensator fit + int8 stage) against
the reference's own FromDenseBoundary (native/src, compiled into
oracle/_ref): K, V, codes, smoothing, scales and the residual, bit for bit."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from gdn_state_codec import codec

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def bits(x):
    return np.ascontiguousarray(x, np.float32).view(np.uint32)


def check(name, got, want):
    got, want = np.asarray(got), np.asarray(want)
    if got.dtype == np.float32:
        bad = int((bits(got) != bits(want)).sum())
    else:
        bad = int((got != want).sum())
    assert bad == 0, f"{name}: {bad} of {got.size} elements differ"


def run_full(dense: np.ndarray, layout: str):
    host = dense if layout == "capsule" else np.ascontiguousarray(dense.transpose(0, 2, 1))
    full = codec.full_encode(torch.from_numpy(host).to(DEV), layout)
    torch.cuda.synchronize()
    flip = (lambda a: a) if layout == "capsule" else (lambda a: a.transpose(0, 2, 1))
    return {
        "codes": flip(full.encoded.codes.cpu().numpy()),
        "smoothing": full.encoded.smoothing.cpu().numpy(),
        "scales": full.encoded.scales.cpu().numpy(),
        "compensator_keys": full.compensator_keys.cpu().numpy(),
        "compensator_values": full.compensator_values.cpu().numpy(),
        "residual": flip(full.residual.cpu().numpy()),
    }


@pytest.mark.parametrize("layout", ["capsule", "provider"])
def test_full_codec_matches_reference_golden(golden, layout):
    g = golden["heads"]
    got = run_full(g["dense"], layout)
    for key in ("compensator_keys", "compensator_values", "codes", "smoothing", "scales"):
        check(key, got[key], g[key])
    residual = np.stack([oracle.rebuild_residual(g["dense"][i], g["compensator_keys"][i],
                                                 g["compensator_values"][i])
                         for i in range(g["dense"].shape[0])])
    check("residual", got["residual"], residual)


def _cases(rng: np.random.Generator) -> np.ndarray:
    heads = []
    for _ in range(8):  # benchmark distribution
        h = (rng.standard_normal((128, 128)) * 10.0 ** (-3.0 * rng.random())).astype(np.float32)
        h[rng.random((128, 128)) < 0.01] = 0.0
        heads.append(h)
    heads.append(np.zeros((128, 128), np.float32))                       # every norm fails
    u, v = rng.standard_normal(128), rng.standard_normal(128)
    heads.append(np.outer(u, v).astype(np.float32))                      # exactly rank 1
    heads.append((rng.standard_normal((128, 128)) * 1e-20).astype(np.float32))  # norms below eps
    one = np.zeros((128, 128), np.float32)
    one[7, 100] = 2.5
    heads.append(one)
    wide = rng.standard_normal((128, 128)) * 10.0 ** rng.uniform(-6, 3, (128, 1))
    heads.append(wide.astype(np.float32))
    return np.stack(heads)


@pytest.mark.skipif(not oracle.ref_available(), reason="reference library not built")
def test_full_codec_matches_live_reference():
    dense = _cases(np.random.default_rng(77))
    want = [oracle.ref_codec_head(dense[i]) for i in range(dense.shape[0])]
    for layout in ("capsule", "provider"):
        got = run_full(dense, layout)
        for key in ("compensator_keys", "compensator_values", "codes", "smoothing", "scales"):
            check(f"{layout} {key}", got[key], np.stack([w[key] for w in want]))


def test_full_codec_reports_non_finite_input():
    dense = torch.zeros((3, 128, 128), device=DEV)
    dense[1, 5, 5] = float("nan")
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    codec.device_error(DEV, clear=True)
    codec.full_encode(dense, "capsule", status=status)
    torch.cuda.synchronize()
    assert int(status.item()) & codec.STATUS_FIT_NON_FINITE
    assert codec.device_error(DEV, clear=True) & codec.STATUS_FIT_NON_FINITE
