"""CPU tests of the C ABI boundary (no GPU needed).

The CUDA library loads on a machine without a GPU, so the boundary itself is
checked here: every entry point declared in include/statecentric/*.h is
exported, the reference's library file names resolve the reference's symbols,
and argument validation (which runs before any CUDA call) rejects what the
reference's launchers reject -- null pointers and zero state counts
(gdn_state_codec_smoothing.cpp:144-146, gdn_state_codec_quantize.cpp:206-210)
-- plus this backend's alignment and layout rules.  No call here reaches the
device: every argument list is one that validation refuses.
"""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from gdn_state_codec import _native

ROOT = Path(__file__).resolve().parents[1]
HEADERS = sorted((ROOT / "include" / "statecentric").glob("*.h"))
PREFIX = "statecentric_gdn_state_codec_"

# Reference symbol -> the library file the reference's loader opens for it
# (src/gdn_state_codec/runtime.py:55-237; ascendc CMakeLists.txt:42,60-61).
REFERENCE_LIBRARIES = {
    "libstatecentric_gdn_state_codec_smoothing_kernel.so": [
        "smoothing_launch_v1", "provider_smoothing_launch_v2"],
    "libstatecentric_gdn_state_codec_quantize_kernel.so": [
        "quantize_launch_v1", "provider_quantize_launch_v2"],
    "libstatecentric_gdn_state_codec_provider_runtime.so": [
        "provider_initialize_launch_v3"],
    "libstatecentric_gdn_state_codec_dequantize_kernel.so": ["dequantize_launch_v1"],
    "libstatecentric_gdn_state_codec_encoded_projection_kernel.so": [
        "encoded_projection_launch_v1", "provider_encoded_projection_launch_v1",
        "encoded_projection_indexed_launch_v1"],
    "libstatecentric_gdn_state_codec_windowed_gdn_step_kernel.so": [
        "windowed_gdn_step_launch_v1", "windowed_gdn_step_bf16_launch_v1",
        "windowed_gdn_step_bf16_quant_only_launch_v1", "fp32_gdn_step_launch_v1"],
    "libstatecentric_gdn_state_codec_window_boundary_kernel.so": [
        "window_boundary_launch_v1"],
    "libstatecentric_gdn_state_codec_bf16_cube_matmul_kernel.so": [],
    "libstatecentric_gdn_state_codec_int8_cube_matmul_kernel.so": [],
}

BAD_ARGS = 1
ALIGNED = 0x10000  # fake, 16-byte aligned, never dereferenced
MISALIGNED = 0x10004


def declared_symbols() -> set[str]:
    names: set[str] = set()
    for header in HEADERS:
        text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
        names.update(re.findall(rf"\b({PREFIX}\w+)\s*\(", text))
    return names


def declared_arity() -> dict[str, int]:
    """Parameter count of every declared entry point."""
    arity: dict[str, int] = {}
    for header in HEADERS:
        text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
        for name, params in re.findall(rf"\b({PREFIX}\w+)\s*\(([^)]*)\)\s*;", text):
            arity[name] = len([p for p in params.split(",") if p.strip()])
    return arity


def lib():
    return _native.load()


def call(name: str, *args) -> int:
    return _native.call(PREFIX + name, *args)


def test_library_loads_without_a_gpu():
    assert _native.library_path().is_file()
    assert lib() is lib()


def test_every_declared_entry_point_is_exported_and_bound():
    names = declared_symbols()
    assert len(names) >= 20
    assert names == set(_native.SIGNATURES), (
        "header declarations and ctypes signatures disagree: "
        f"{sorted(names ^ set(_native.SIGNATURES))}")
    for name in names:
        assert hasattr(lib(), name), name
    arity = declared_arity()
    assert set(arity) == names
    for name, argtypes in _native.SIGNATURES.items():
        assert len(argtypes) == arity[name], (name, len(argtypes), arity[name])


@pytest.mark.parametrize("library", sorted(REFERENCE_LIBRARIES))
def test_reference_library_names_resolve(library):
    """A loader written for the reference finds its symbols under the
    reference's file names (the files depend on the core library)."""
    path = _native.library_dir() / library
    assert path.is_file(), path
    handle = ctypes.CDLL(str(path))
    for symbol in REFERENCE_LIBRARIES[library]:
        assert hasattr(handle, PREFIX + symbol), (library, symbol)


def test_null_pointers_and_zero_states_are_rejected():
    n = None
    a = ALIGNED
    # reference single-head entry points: any null pointer
    assert call("smoothing_launch_v1", n, n, a) == BAD_ARGS
    assert call("smoothing_launch_v1", n, a, n) == BAD_ARGS
    assert call("quantize_launch_v1", n, a, a, a, n) == BAD_ARGS
    assert call("dequantize_launch_v1", n, a, a, a, a, a, n) == BAD_ARGS
    # the reference's single-head dequantize needs both compensators
    assert call("dequantize_launch_v1", n, a, a, a, n, n, a) == BAD_ARGS
    # batched entry points: null pointers and states == 0
    for name in ("provider_smoothing_launch_v2",):
        assert call(name, n, a, a, 0) == BAD_ARGS
        assert call(name, n, n, a, 1) == BAD_ARGS
    for name in ("provider_quantize_launch_v2", "provider_initialize_launch_v3",
                 "initialize_launch_v3"):
        assert call(name, n, a, a, a, a, 0) == BAD_ARGS
        assert call(name, n, a, a, n, a, 4) == BAD_ARGS
    for name in ("dequantize_launch_v2", "provider_dequantize_launch_v2"):
        assert call(name, n, a, a, a, n, n, a, 0) == BAD_ARGS
        assert call(name, n, a, a, a, n, n, n, 4) == BAD_ARGS
        # compensators come in pairs
        assert call(name, n, a, a, a, a, n, a, 4) == BAD_ARGS
        assert call(name, n, a, a, a, n, a, a, 4) == BAD_ARGS
    for name in ("encoded_projection_launch_v1", "provider_encoded_projection_launch_v1"):
        assert call(name, n, a, a, a, n, n, a, a, 0) == BAD_ARGS
        assert call(name, n, a, a, a, n, n, n, a, 4) == BAD_ARGS
        assert call(name, n, a, a, a, a, n, a, a, 4) == BAD_ARGS


def test_misaligned_buffers_are_rejected():
    a, m, n = ALIGNED, MISALIGNED, None
    assert call("initialize_launch_v3", n, m, a, a, a, 1) == BAD_ARGS
    assert call("provider_initialize_launch_v3", n, a, a, a, m, 1) == BAD_ARGS
    assert call("dequantize_launch_v2", n, a, a, a, n, n, m, 1) == BAD_ARGS
    # queries need 8-byte alignment, outputs 16
    assert call("encoded_projection_launch_v1", n, a, a, a, n, n, a + 2, a, 1) == BAD_ARGS
    assert call("encoded_projection_launch_v1", n, a, a, a, n, n, a, a + 8, 1) == BAD_ARGS


def test_indexed_geometry_is_validated():
    a, n = ALIGNED, None
    # layout must be 0 (capsule) or 1 (provider)
    assert call("initialize_indexed_launch_v1", n, 2, a, a, a, a, a, 4, 32, 8, n) == BAD_ARGS
    # slot ids required, int32-aligned; count, heads_per_slot, num_slots >= 1
    assert call("initialize_indexed_launch_v1", n, 0, a, a, a, a, n, 4, 32, 8, n) == BAD_ARGS
    assert call("initialize_indexed_launch_v1", n, 0, a, a, a, a, a + 1, 4, 32, 8, n) == BAD_ARGS
    assert call("initialize_indexed_launch_v1", n, 0, a, a, a, a, a, 0, 32, 8, n) == BAD_ARGS
    assert call("dequantize_indexed_launch_v1", n, 1, a, a, a, n, n, a, a, 4, 0, 8, n) == BAD_ARGS
    assert call("dequantize_indexed_launch_v1", n, 1, a, a, a, a, n, a, a, 4, 32, 8, n) == BAD_ARGS
    assert call("encoded_projection_indexed_launch_v1",
                n, 0, a, a, a, n, n, a, a, a, 4, 32, 0, n) == BAD_ARGS


def test_full_codec_entry_point_validates():
    a, n = ALIGNED, None
    assert call("full_initialize_launch_v1", n, 2, a, a, a, a, a, a, a, 1, n) == BAD_ARGS
    assert call("full_initialize_launch_v1", n, 0, a, a, a, a, a, a, a, 0, n) == BAD_ARGS
    assert call("full_initialize_launch_v1", n, 0, a, n, a, a, a, a, a, 1, n) == BAD_ARGS
    assert call("full_initialize_launch_v1", n, 1, a, a, a, a, a, a, MISALIGNED, 1, n) == BAD_ARGS


def test_status_and_support_entry_points_validate():
    assert call("device_error_v1", None, 0) == BAD_ARGS
    assert call("synthesize_states_v1", None, None, 0, 0, 0, 1, 1, 1) == BAD_ARGS
    assert call("synthesize_states_v1", None, ALIGNED, 2, 0, 0, 1, 1, 1) == BAD_ARGS
    assert call("synthesize_queries_v1", None, ALIGNED, 0, 0, 0, 1, 1) == BAD_ARGS
    assert call("division_selftest_v1", None, None, ALIGNED, ALIGNED, 1) == BAD_ARGS


def test_wait_selftest_entry_points_validate():
    """The failure-path test launchers refuse a missing status word, a zero
    or over-long limit and the batched launchers' bad arguments."""
    a, m, n = ALIGNED, MISALIGNED, None
    q = "quantize_wait_selftest_v1"
    assert call(q, n, a, a, a, a, 1, 1000, n) == BAD_ARGS           # no status word
    assert call(q, n, a, a, a, a, 1, 0, a) == BAD_ARGS              # zero limit
    assert call(q, n, a, a, a, a, 1, 2_000_000_001, a) == BAD_ARGS  # longer than 2 s
    assert call(q, n, a, a, a, a, 0, 1000, a) == BAD_ARGS           # no states
    assert call(q, n, m, a, a, a, 1, 1000, a) == BAD_ARGS           # misaligned state
    p = "encoded_projection_wait_selftest_v1"
    assert call(p, n, a, a, a, a, a, 1, 1000, n) == BAD_ARGS
    assert call(p, n, a, a, a, a, a, 1, 0, a) == BAD_ARGS
    assert call(p, n, a, a, a, n, a, 1, 1000, a) == BAD_ARGS        # no queries
    assert call(p, n, a, a, a, a, a, 0, 1000, a) == BAD_ARGS
    d = "fp32_gdn_step_wait_selftest_v1"
    assert call(d, n, a, a, a, a, a, a, a, 1, 0) == BAD_ARGS            # zero limit
    assert call(d, n, a, a, a, a, a, a, a, 1, 2_000_000_001) == BAD_ARGS
    assert call(d, n, a, a, a, a, a, a, a, 0, 1000) == BAD_ARGS         # no states
    assert call(d, n, m, a, a, a, a, a, a, 1, 1000) == BAD_ARGS         # misaligned state


def _window(a=ALIGNED):
    # codes, smoothing, scales, compensator keys / values, record decay /
    # keys / corrections, positions
    return [a] * 9


def test_windowed_decode_entry_points_validate():
    """The window launchers refuse what the reference's refuse (null
    pointers, zero states, odd states for the bf16 step, more than 32 power
    iterations) plus this backend's alignment rules."""
    a, m, n = ALIGNED, MISALIGNED, None
    token = [a] * 5 + [a]  # decay, beta / keys, queries..., outputs
    step_bf16 = ["windowed_gdn_step_bf16_launch_v1",
                 "windowed_gdn_step_bf16_quant_only_launch_v1"]
    for name in step_bf16:
        assert call(name, n, *_window(), *token, 0) == BAD_ARGS            # no states
        assert call(name, n, *_window(), *token, 3) == BAD_ARGS            # odd states
        assert call(name, n, *([n] + _window()[1:]), *token, 2) == BAD_ARGS  # no codes
        assert call(name, n, *([a + 8] + _window()[1:]), *token, 2) == BAD_ARGS  # codes misaligned
        assert call(name, n, *_window(), *token[:5], n, 2) == BAD_ARGS     # no outputs
    # compensators: required by the full step, optional for quant-only, paired
    w = _window()
    w[3] = w[4] = n
    assert call(step_bf16[0], n, *w, *token, 2) == BAD_ARGS
    w = _window()
    w[4] = n
    assert call(step_bf16[1], n, *w, *token, 2) == BAD_ARGS
    w = _window()
    w[3] = a + 8  # compensators must be 16-byte aligned
    assert call(step_bf16[0], n, *w, *token, 2) == BAD_ARGS
    assert call("windowed_gdn_step_launch_v1", n, *_window(), *token, 0) == BAD_ARGS
    assert call("windowed_gdn_step_launch_v1", n, *_window(), m + 1, *token[1:], 1) == BAD_ARGS
    boundary = _window() + [a] * 6  # next codes / smoothing / scales / keys / values, workspace
    assert call("window_boundary_launch_v1", n, *boundary, 1, 33) == BAD_ARGS
    assert call("window_boundary_launch_v1", n, *boundary, 0, 0) == BAD_ARGS
    assert call("window_boundary_launch_v1", n, *boundary[:-1], m, 1, 0) == BAD_ARGS
    assert call("fp32_gdn_step_launch_v1", n, a, a, a, a, a, a, a, 0) == BAD_ARGS
    assert call("fp32_gdn_step_launch_v1", n, n, a, a, a, a, a, a, 1) == BAD_ARGS
    # the dense state is staged by bulk copies: 16-byte alignment required
    assert call("fp32_gdn_step_launch_v1", n, a + 4, a, a, a, a, a, a, 1) == BAD_ARGS


def test_valid_arguments_without_a_device_report_setup_failure():
    """With no CUDA device the launchers return 3 (set-up failed) instead of
    crashing: the product has no CPU fallback."""
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present; fake pointers must not reach it")
    a = ALIGNED
    assert call("initialize_launch_v3", None, a, a, a, a, 1) == 3
    assert call("provider_dequantize_launch_v2", None, a, a, a, None, None, a, 1) == 3
    assert call("windowed_gdn_step_bf16_launch_v1", None, *_window(), *([a] * 6), 2) == 3


def test_headers_compile_as_c_and_link(tmp_path):
    """A C caller (the reference's C ABI has no C++ types) includes both
    headers, links the core library and gets 1 from a launcher given null
    pointers, which validation refuses before any CUDA call."""
    import shutil
    import subprocess

    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    source = tmp_path / "caller.c"
    source.write_text(
        '#include "statecentric/gdn_state_codec_kernel.h"\n'
        '#include "statecentric/gdn_state_codec_windowed_gdn_kernel.h"\n'
        "int main(void) {\n"
        "  int32_t status = statecentric_gdn_state_codec_provider_initialize_launch_v3(\n"
        "      (void*)0, (const float*)0, (float*)0, (int8_t*)0, (float*)0, 1u);\n"
        "  int32_t window = statecentric_gdn_state_codec_fp32_gdn_step_launch_v1(\n"
        "      (void*)0, (float*)0, (const float*)0, (const uint16_t*)0, (const uint16_t*)0,\n"
        "      (const uint16_t*)0, (const uint16_t*)0, (float*)0, 1u);\n"
        "  return status == 1 && window == 1 ? 0 : 1;\n"
        "}\n")
    lib_dir = Path(_native.DEFAULT_LIBRARY_DIR)
    exe = tmp_path / "caller"
    subprocess.run([cc, "-std=c11", "-Wall", "-Wextra", "-Werror", "-pedantic",
                    f"-I{ROOT / 'include'}", str(source), "-o", str(exe), f"-L{lib_dir}",
                    f"-l:{_native.CORE_LIBRARY}", f"-Wl,-rpath,{lib_dir}"],
                   check=True, capture_output=True, text=True)
    assert subprocess.run([str(exe)], timeout=60).returncode == 0
