# SPDX-License-Identifier: Apache-2.0
"""Fail-closed activation contract of the GDN state codec (CUDA / B200).

Mirrors the reference's src/gdn_state_codec/config.py:1-101: the same
``additional_config.gdn_state_codec`` keys, value ranges and error messages,
with one change -- the device gate admits CUDA (B200, sm_100a) instead of
Ascend NPU (config.py:84-85).
"""

from __future__ import annotations

import os
from dataclasses import dataclass
from pathlib import Path
from typing import Any

_QWEN35_GENERATION_ARCHITECTURES = frozenset(
    {
        "Qwen3_5ForConditionalGeneration",
        "Qwen3_5MoeForConditionalGeneration",
    }
)
SUPPORTED_DEVICE_TYPE = "cuda"


@dataclass(frozen=True, slots=True)
class GdnStateCodecExperiment:
    library_dir: Path
    mode: str
    initializer: str
    boundary_power_iterations: int
    decode_backend: str


def parse_gdn_state_codec_experiment(
    additional_config: dict[str, Any] | object,
    architectures: list[str] | tuple[str, ...],
    device_type: str,
    enforce_eager: bool,
    speculative_method: str | None,
    num_speculative_tokens: int,
) -> GdnStateCodecExperiment | None:
    """Validate the experiment configuration before any native code loads.

    Returns None when the experiment is not configured; raises ValueError on
    any configuration the codec does not admit."""
    if not isinstance(additional_config, dict):
        return None
    raw = additional_config.get("gdn_state_codec")
    if raw is None:
        return None
    expected = {"initializer", "boundary_power_iterations", "decode_backend", "mode"}
    if not isinstance(raw, dict) or set(raw) != expected:
        raise ValueError(
            "gdn_state_codec must contain exactly boundary_power_iterations, "
            "decode_backend, initializer, and mode"
        )

    library_dir = os.environ.get("GDN_STATE_CODEC_LIBRARY_DIR", "")
    library_path = Path(library_dir)
    if not library_dir or not library_path.is_absolute():
        raise ValueError(
            "GDN_STATE_CODEC_LIBRARY_DIR must name an absolute native-library directory"
        )

    mode = raw["mode"]
    initializer = raw["initializer"]
    iterations = raw["boundary_power_iterations"]
    decode_backend = raw["decode_backend"]
    if mode not in {"shadow", "replace"}:
        raise ValueError("gdn_state_codec.mode must be 'shadow' or 'replace'")
    if initializer not in {"exact_svd", "quant_only"}:
        raise ValueError("gdn_state_codec.initializer must be 'exact_svd' or 'quant_only'")
    if decode_backend not in {"vector", "cube"}:
        raise ValueError("gdn_state_codec.decode_backend must be 'vector' or 'cube'")
    if (
        not isinstance(iterations, int)
        or isinstance(iterations, bool)
        or not 0 <= iterations <= 32
        or (iterations == 0 and initializer != "quant_only")
    ):
        raise ValueError(
            "gdn_state_codec.boundary_power_iterations must be in [1,32], "
            "or 0 with quant_only initialization"
        )
    if device_type != SUPPORTED_DEVICE_TYPE:
        raise ValueError("gdn_state_codec only supports CUDA (B200, sm_100a)")
    if not set(architectures).intersection(_QWEN35_GENERATION_ARCHITECTURES):
        raise ValueError("gdn_state_codec only supports Qwen3.5 generation models")
    if not enforce_eager:
        raise ValueError("gdn_state_codec currently requires enforce_eager")
    if speculative_method is not None or num_speculative_tokens != 0:
        raise ValueError("gdn_state_codec currently excludes speculative decoding")
    return GdnStateCodecExperiment(
        library_dir=library_path,
        mode=mode,
        initializer=initializer,
        boundary_power_iterations=iterations,
        decode_backend=decode_backend,
    )


__all__ = ["GdnStateCodecExperiment", "parse_gdn_state_codec_experiment"]
