"""Build the B200 GDN state codec libraries in-tree (no GPU needed).

Outputs, all under ``lib/`` next to this file:

* ``libgdn_state_codec_b200.so`` -- every kernel and the C ABI of
  ``include/statecentric/gdn_state_codec_kernel.h``, compiled by nvcc for
  sm_100a only (``-gencode arch=compute_100a,code=sm_100a``).
* the reference's library file names (``libstatecentric_gdn_state_codec_*``,
  see ``NAMED_LIBRARIES``): thin files that depend on the library above, so a
  loader written for the reference (src/gdn_state_codec/runtime.py:55-237)
  finds every entry point under the names it expects.

Compile flags that carry the arithmetic contract: ``-fmad=false`` (nvcc never
contracts a multiply and an add into an FMA on its own) and the default
IEEE-rounded division and square root (no ``--use_fast_math``).
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
REPO_ROOT = PACKAGE_DIR.parent
CSRC = PACKAGE_DIR / "csrc"
INCLUDE = REPO_ROOT / "include"
LIB_DIR = PACKAGE_DIR / "lib"
CORE_NAME = "libgdn_state_codec_b200.so"
CORE_LIB = LIB_DIR / CORE_NAME

# Library file names the reference's plugin loads (runtime.py:55-76, 100-106,
# 130-134, 153-154, 180-183, 200-203, 222-225) plus the dequantize library of
# native/ascendc/gdn_state_codec/CMakeLists.txt:42.
NAMED_LIBRARIES = (
    "libstatecentric_gdn_state_codec_smoothing_kernel.so",
    "libstatecentric_gdn_state_codec_quantize_kernel.so",
    "libstatecentric_gdn_state_codec_dequantize_kernel.so",
    "libstatecentric_gdn_state_codec_provider_runtime.so",
    "libstatecentric_gdn_state_codec_encoded_projection_kernel.so",
    "libstatecentric_gdn_state_codec_windowed_gdn_step_kernel.so",
    "libstatecentric_gdn_state_codec_window_boundary_kernel.so",
    "libstatecentric_gdn_state_codec_bf16_cube_matmul_kernel.so",
    "libstatecentric_gdn_state_codec_int8_cube_matmul_kernel.so",
)

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-fmad=false",
    "-Xcompiler", "-fPIC,-fvisibility=default",
    "-Xptxas", "-warn-spills",
    "-diag-suppress", "550",
]


def _nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    candidate = Path(cuda_home) / "bin" / "nvcc"
    if candidate.is_file():
        return str(candidate)
    found = shutil.which("nvcc")
    if found is None:
        raise RuntimeError("nvcc not found: the B200 codec needs the CUDA toolkit to build")
    return found


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted(
        INCLUDE.glob("statecentric/*.h"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.is_file():
        return True
    built = target.stat().st_mtime
    return any(dep.stat().st_mtime > built for dep in deps)


def _run(cmd: list[str]) -> None:
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        sys.stderr.write(result.stdout + result.stderr)
        raise RuntimeError(f"build step failed ({result.returncode}): {' '.join(cmd)}")


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile the core library and the named libraries; returns LIB_DIR."""
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    if force or _stale(CORE_LIB, _sources()):
        cmd = [_nvcc(), *NVCC_FLAGS, "-shared", f"-I{INCLUDE}", f"-I{CSRC}",
               str(CSRC / "gdn_state_codec.cu"), "-o", str(CORE_LIB)]
        if verbose:
            print(" ".join(cmd))
        _run(cmd)
    shim_src = CSRC / "named_library.c"
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        raise RuntimeError("no C compiler found for the named libraries")
    for name in NAMED_LIBRARIES:
        target = LIB_DIR / name
        if force or _stale(target, [shim_src, CORE_LIB]):
            _run([cc, "-shared", "-fPIC", "-O2", "-o", str(target), str(shim_src),
                  f"-L{LIB_DIR}", "-Wl,--no-as-needed", f"-l:{CORE_NAME}",
                  "-Wl,-rpath,$ORIGIN"])
    return LIB_DIR


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(f"built {CORE_LIB} and {len(NAMED_LIBRARIES)} named libraries")
