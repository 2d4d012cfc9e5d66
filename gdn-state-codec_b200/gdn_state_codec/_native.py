# SPDX-License-Identifier: Apache-2.0
"""ctypes binding of the B200 codec's C ABI (include/statecentric/*.h).

The library is loaded from ``GDN_STATE_CODEC_LIBRARY_DIR`` when set, else
from ``lib/`` beside this package (where ``build.py`` puts it).  There is no
fallback: when the CUDA library is missing every call raises.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

PACKAGE_ROOT = Path(__file__).resolve().parent.parent
DEFAULT_LIBRARY_DIR = PACKAGE_ROOT / "lib"
CORE_LIBRARY = "libgdn_state_codec_b200.so"

_vp = ctypes.c_void_p
_u32 = ctypes.c_uint32
_u64 = ctypes.c_uint64
_i32 = ctypes.c_int32

# name -> argument types (every entry point returns int32 status).
SIGNATURES: dict[str, list] = {
    # reference entry points (gdn_state_codec_kernel.h:5-36)
    "statecentric_gdn_state_codec_smoothing_launch_v1": [_vp, _vp, _vp],
    "statecentric_gdn_state_codec_provider_smoothing_launch_v2": [_vp, _vp, _vp, _u32],
    "statecentric_gdn_state_codec_quantize_launch_v1": [_vp, _vp, _vp, _vp, _vp],
    "statecentric_gdn_state_codec_provider_quantize_launch_v2": [_vp] * 5 + [_u32],
    "statecentric_gdn_state_codec_provider_initialize_launch_v3": [_vp] * 5 + [_u32],
    "statecentric_gdn_state_codec_dequantize_launch_v1": [_vp] * 7,
    # batched extensions
    "statecentric_gdn_state_codec_initialize_launch_v3": [_vp] * 5 + [_u32],
    "statecentric_gdn_state_codec_dequantize_launch_v2": [_vp] * 7 + [_u32],
    "statecentric_gdn_state_codec_provider_dequantize_launch_v2": [_vp] * 7 + [_u32],
    "statecentric_gdn_state_codec_encoded_projection_launch_v1": [_vp] * 8 + [_u32],
    "statecentric_gdn_state_codec_provider_encoded_projection_launch_v1": [_vp] * 8 + [_u32],
    # slot-indexed extensions
    "statecentric_gdn_state_codec_initialize_indexed_launch_v1":
        [_vp, _u32] + [_vp] * 5 + [_u32, _u32, _u32, _vp],
    "statecentric_gdn_state_codec_dequantize_indexed_launch_v1":
        [_vp, _u32] + [_vp] * 7 + [_u32, _u32, _u32, _vp],
    "statecentric_gdn_state_codec_encoded_projection_indexed_launch_v1":
        [_vp, _u32] + [_vp] * 8 + [_u32, _u32, _u32, _vp],
    # full codec (rank-4 fit + int8 stage)
    "statecentric_gdn_state_codec_full_initialize_launch_v1":
        [_vp, _u32] + [_vp] * 7 + [_u32, _vp],
    "statecentric_gdn_state_codec_full_initialize_static_launch_v1":
        [_vp, _u32] + [_vp] * 6 + [_u32, _vp],
    # capsule wire format
    "statecentric_gdn_state_codec_capsule_serialize_launch_v1":
        [_vp, _u32] + [_vp] * 6 + [_u64, _u64, _vp, _u32],
    "statecentric_gdn_state_codec_capsule_restore_launch_v1":
        [_vp, _u32, _vp, _vp, _u64, _u64] + [_vp] * 6 + [_u32],
    "statecentric_gdn_state_codec_sha256_v1": [_vp, _u64, _vp],
    # status and benchmark support
    "statecentric_gdn_state_codec_device_error_v1": [_vp, _i32],
    "statecentric_gdn_state_codec_synthesize_states_v1":
        [_vp, _vp, _u32, _u64, _u32, _u32, _u32, _u32],
    "statecentric_gdn_state_codec_synthesize_queries_v1":
        [_vp, _vp, _u64, _u32, _u32, _u32, _u32],
    "statecentric_gdn_state_codec_division_selftest_v1": [_vp, _vp, _vp, _vp, _u64],
    "statecentric_gdn_state_codec_quantize_wait_selftest_v1": [_vp] * 5 + [_u32, _u64, _vp],
    "statecentric_gdn_state_codec_fp32_gdn_step_wait_selftest_v1": [_vp] * 8 + [_u32, _u64],
    "statecentric_gdn_state_codec_encoded_projection_wait_selftest_v1":
        [_vp] * 6 + [_u32, _u64, _vp],
    # windowed decode (gdn_state_codec_windowed_gdn_kernel.h)
    "statecentric_gdn_state_codec_windowed_gdn_step_launch_v1": [_vp] * 16 + [_u32],
    "statecentric_gdn_state_codec_windowed_gdn_step_bf16_launch_v1": [_vp] * 16 + [_u32],
    "statecentric_gdn_state_codec_windowed_gdn_step_bf16_quant_only_launch_v1":
        [_vp] * 16 + [_u32],
    "statecentric_gdn_state_codec_window_boundary_launch_v1": [_vp] * 16 + [_u32, _u32],
    "statecentric_gdn_state_codec_fp32_gdn_step_launch_v1": [_vp] * 8 + [_u32],
}

_lock = threading.Lock()
_library: ctypes.CDLL | None = None


def library_dir() -> Path:
    configured = os.environ.get("GDN_STATE_CODEC_LIBRARY_DIR", "")
    return Path(configured) if configured else DEFAULT_LIBRARY_DIR


def library_path() -> Path:
    return library_dir() / CORE_LIBRARY


def load() -> ctypes.CDLL:
    """Load the CUDA library once and bind every entry point's signature."""
    global _library
    with _lock:
        if _library is not None:
            return _library
        path = library_path()
        if not path.is_file():
            raise RuntimeError(
                f"GDN State Codec B200 library is missing: {path} "
                "(build it with gdn-state-codec_b200/build.py)"
            )
        handle = ctypes.CDLL(str(path))
        for name, argtypes in SIGNATURES.items():
            function = getattr(handle, name)
            function.argtypes = argtypes
            function.restype = _i32
        _library = handle
        return handle


def call(name: str, *args) -> int:
    return int(getattr(load(), name)(*args))
