"""Shared pytest set-up: import paths, the ``gpu`` marker, common fixtures."""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for path in (ROOT / "gdn-state-codec_b200", ROOT / "oracle", ROOT):
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))

GOLDEN = Path(__file__).resolve().parent / "golden"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (runs on the B200 box)")


@pytest.fixture(scope="session")
def golden():
    import numpy as np

    return {
        "heads": dict(np.load(GOLDEN / "reference_heads.npz")),
        "small": dict(np.load(GOLDEN / "reference_small.npz")),
        "adapter": dict(np.load(GOLDEN / "adapter.npz")),
        "quant_only": dict(np.load(GOLDEN / "reference_quant_only.npz")),
    }
