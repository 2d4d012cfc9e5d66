"""CPU oracle for the GDN state codec hot path -- TEST INFRASTRUCTURE ONLY.

Thin numpy/ctypes front end over ``liboracle.so`` (the C restatement in
``gdn_codec_oracle.c``) and, when it has been built in this container, over
``_ref/libgdn_ref.so`` (the reference's own portable library from
native/src of vLLM-HUST/gdn-state-codec, wrapped by ``ref_shim.cpp``).

Only tests/, ``__graft_entry__.smoke()`` and the CPU-baseline legs of
``bench.py`` import this module, and only as the checker; the product
library never routes through it.

Layouts (one head = one [128,128] GDN state matrix):
  capsule  [key, value]  -- native/src capsule layout, BASELINE's [H, d_k, d_v]
  provider [value, key]  -- vLLM's ssm_state layout (runtime.py:460-471)
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
LIB_PATH = ORACLE_DIR / "liboracle.so"
REF_LIB_PATH = ORACLE_DIR / "_ref" / "libgdn_ref.so"
RANK = 4

_lib = None
_ref = None

_f32p = ctypes.POINTER(ctypes.c_float)
_i8p = ctypes.POINTER(ctypes.c_int8)


def _ptr(array: np.ndarray | None, ctype):
    if array is None:
        return ctypes.cast(None, ctype)
    assert array.flags["C_CONTIGUOUS"]
    return array.ctypes.data_as(ctype)


def build() -> None:
    """Compile liboracle.so (and _ref/ when the reference tree is present)."""
    import subprocess

    subprocess.run(["make", "-s", "-C", str(ORACLE_DIR)], check=True)
    # GDN_REFERENCE_ROOT when set, else a directory `reference` beside the repo.
    ref_root = Path(os.environ.get("GDN_REFERENCE_ROOT", ORACLE_DIR.parent.parent / "reference"))
    if (ref_root / "native" / "src").is_dir():
        subprocess.run(
            ["make", "-s", "-C", str(ORACLE_DIR), "ref", f"REF={ref_root}"],
            check=True,
        )


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.is_file():
            raise RuntimeError(f"oracle library not built: {LIB_PATH}")
        handle = ctypes.CDLL(str(LIB_PATH))
        u64, u32, c_int = ctypes.c_uint64, ctypes.c_uint32, ctypes.c_int
        handle.oracle_smoothing.argtypes = [_f32p, u64, u32, u32, c_int, _f32p]
        handle.oracle_quantize_given_smoothing.argtypes = [
            _f32p, _f32p, u64, u32, u32, c_int, _i8p, _f32p]
        handle.oracle_quantize.argtypes = [
            _f32p, u64, u32, u32, c_int, _f32p, _i8p, _f32p]
        handle.oracle_dequantize.argtypes = [
            _i8p, _f32p, _f32p, _f32p, _f32p, u64, u32, u32, c_int, _f32p]
        handle.oracle_project.argtypes = [
            _i8p, _f32p, _f32p, _f32p, _f32p, _f32p, u64, u32, u32, c_int, _f32p]
        handle.oracle_provider_to_capsule.argtypes = [_f32p, u64, u32, u32, _f32p]
        handle.oracle_capsule_to_provider.argtypes = [_f32p, u64, u32, u32, _f32p]
        handle.oracle_quantize_mt.argtypes = [
            _f32p, u64, u32, u32, c_int, _f32p, _i8p, _f32p, c_int]
        handle.oracle_quantize_mt.restype = c_int
        handle.oracle_dequantize_mt.argtypes = [
            _i8p, _f32p, _f32p, u64, u32, u32, c_int, _f32p, c_int]
        handle.oracle_dequantize_mt.restype = c_int
        handle.oracle_project_mt.argtypes = [
            _i8p, _f32p, _f32p, _f32p, u64, u32, u32, c_int, _f32p, c_int]
        handle.oracle_project_mt.restype = c_int
        _lib = handle
    return _lib


def _geometry(state: np.ndarray, layout: str) -> tuple[int, int, int, int]:
    if state.ndim != 3:
        raise ValueError("expected [heads, rows, cols]")
    heads, rows, cols = state.shape
    provider = 1 if layout == "provider" else 0
    keys, values = (cols, rows) if provider else (rows, cols)
    return heads, keys, values, provider


def smoothing(state: np.ndarray, layout: str = "capsule") -> np.ndarray:
    state = np.ascontiguousarray(state, dtype=np.float32)
    heads, keys, values, provider = _geometry(state, layout)
    c = np.empty((heads, keys), np.float32)
    lib().oracle_smoothing(_ptr(state, _f32p), heads, keys, values, provider,
                           _ptr(c, _f32p))
    return c


def quantize(state: np.ndarray, layout: str = "capsule", smoothing_in=None,
             threads: int = 1):
    """Fused smoothing + quantize: returns (codes, smoothing, scales).

    With ``smoothing_in`` the smoothing is taken as given (the reference's
    quantize_launch_v1 / provider_quantize_launch_v2 contract)."""
    state = np.ascontiguousarray(state, dtype=np.float32)
    heads, keys, values, provider = _geometry(state, layout)
    codes = np.empty(state.shape, np.int8)
    b = np.empty((heads, values), np.float32)
    if smoothing_in is not None:
        c = np.ascontiguousarray(smoothing_in, dtype=np.float32).reshape(heads, keys)
        lib().oracle_quantize_given_smoothing(
            _ptr(state, _f32p), _ptr(c, _f32p), heads, keys, values, provider,
            _ptr(codes, _i8p), _ptr(b, _f32p))
        return codes, c, b
    c = np.empty((heads, keys), np.float32)
    if threads > 1:
        lib().oracle_quantize_mt(_ptr(state, _f32p), heads, keys, values, provider,
                                 _ptr(c, _f32p), _ptr(codes, _i8p), _ptr(b, _f32p),
                                 threads)
    else:
        lib().oracle_quantize(_ptr(state, _f32p), heads, keys, values, provider,
                              _ptr(c, _f32p), _ptr(codes, _i8p), _ptr(b, _f32p))
    return codes, c, b


def dequantize(codes, c, b, compensator_keys=None, compensator_values=None,
               layout: str = "capsule", threads: int = 1) -> np.ndarray:
    codes = np.ascontiguousarray(codes, dtype=np.int8)
    heads, keys, values, provider = _geometry(codes, layout)
    c = np.ascontiguousarray(c, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    out = np.empty(codes.shape, np.float32)
    if threads > 1 and compensator_keys is None:
        lib().oracle_dequantize_mt(_ptr(codes, _i8p), _ptr(c, _f32p), _ptr(b, _f32p),
                                   heads, keys, values, provider, _ptr(out, _f32p),
                                   threads)
        return out
    ck = None if compensator_keys is None else np.ascontiguousarray(
        compensator_keys, dtype=np.float32)
    cv = None if compensator_values is None else np.ascontiguousarray(
        compensator_values, dtype=np.float32)
    lib().oracle_dequantize(_ptr(codes, _i8p), _ptr(c, _f32p), _ptr(b, _f32p),
                            _ptr(ck, _f32p), _ptr(cv, _f32p), heads, keys, values,
                            provider, _ptr(out, _f32p))
    return out


def project(codes, c, b, queries, compensator_keys=None, compensator_values=None,
            layout: str = "capsule", threads: int = 1) -> np.ndarray:
    """Encoded projection o[h, v] = (dequant(S_h)^T q_h)[v] from the codes."""
    codes = np.ascontiguousarray(codes, dtype=np.int8)
    heads, keys, values, provider = _geometry(codes, layout)
    c = np.ascontiguousarray(c, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    x = np.ascontiguousarray(queries, dtype=np.float32).reshape(heads, keys)
    out = np.empty((heads, values), np.float32)
    if threads > 1 and compensator_keys is None:
        lib().oracle_project_mt(_ptr(codes, _i8p), _ptr(c, _f32p), _ptr(b, _f32p),
                                _ptr(x, _f32p), heads, keys, values, provider,
                                _ptr(out, _f32p), threads)
        return out
    ck = None if compensator_keys is None else np.ascontiguousarray(
        compensator_keys, dtype=np.float32)
    cv = None if compensator_values is None else np.ascontiguousarray(
        compensator_values, dtype=np.float32)
    lib().oracle_project(_ptr(codes, _i8p), _ptr(c, _f32p), _ptr(b, _f32p),
                         _ptr(ck, _f32p), _ptr(cv, _f32p), _ptr(x, _f32p), heads,
                         keys, values, provider, _ptr(out, _f32p))
    return out


def provider_to_capsule(provider: np.ndarray) -> np.ndarray:
    provider = np.ascontiguousarray(provider, dtype=np.float32)
    heads, values, keys = provider.shape
    out = np.empty((heads, keys, values), np.float32)
    lib().oracle_provider_to_capsule(_ptr(provider, _f32p), heads, keys, values,
                                     _ptr(out, _f32p))
    return out


def capsule_to_provider(capsule: np.ndarray) -> np.ndarray:
    capsule = np.ascontiguousarray(capsule, dtype=np.float32)
    heads, keys, values = capsule.shape
    out = np.empty((heads, values, keys), np.float32)
    lib().oracle_capsule_to_provider(_ptr(capsule, _f32p), heads, keys, values,
                                     _ptr(out, _f32p))
    return out


def rebuild_residual(dense: np.ndarray, compensator_keys: np.ndarray,
                     compensator_values: np.ndarray) -> np.ndarray:
    """Residual left after the reference's rank-4 fit, capsule.cpp:182-187.

    The reference subtracts ``left * sv * right`` rank by rank; it stores
    ``left * sv`` as the compensator key, so the same fp32 products
    (K[k,r] * V[v,r], then one subtraction, no FMA) rebuild R exactly."""
    r = np.array(dense, dtype=np.float32, copy=True)
    ck = np.asarray(compensator_keys, np.float32)
    cv = np.asarray(compensator_values, np.float32)
    keys, values = r.shape
    ck = ck.reshape(keys, RANK)
    cv = cv.reshape(values, RANK)
    for rank in range(RANK):
        r -= np.outer(ck[:, rank], cv[:, rank]).astype(np.float32)
    return r


# --------------------------------------------------------------------------
# The reference library itself (only where it was compiled from source here).

def ref_available() -> bool:
    return REF_LIB_PATH.is_file()


def ref() -> ctypes.CDLL:
    global _ref
    if _ref is None:
        if not REF_LIB_PATH.is_file():
            raise RuntimeError(f"reference library not built: {REF_LIB_PATH}")
        handle = ctypes.CDLL(str(REF_LIB_PATH))
        u32 = ctypes.c_uint32
        handle.ref_codec_head.argtypes = [
            _f32p, u32, u32, _f32p, _i8p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p]
        handle.ref_codec_head.restype = ctypes.c_int
        handle.ref_provider_to_capsule.argtypes = [_f32p, u32, u32, _f32p]
        handle.ref_provider_to_capsule.restype = ctypes.c_int
        handle.ref_head_bytes.argtypes = [
            u32, u32, ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint64)]
        handle.ref_head_bytes.restype = ctypes.c_int
        _ref = handle
    return _ref


def ref_codec_head(dense: np.ndarray, query: np.ndarray | None = None) -> dict:
    """Run the real reference codec on one capsule-layout head."""
    dense = np.ascontiguousarray(dense, dtype=np.float32)
    keys, values = dense.shape
    out = {
        "codes": np.empty((keys, values), np.int8),
        "smoothing": np.empty(keys, np.float32),
        "scales": np.empty(values, np.float32),
        "compensator_keys": np.empty((keys, RANK), np.float32),
        "compensator_values": np.empty((values, RANK), np.float32),
        "dense_state": np.empty((keys, values), np.float32),
        "projection": np.empty(values, np.float32),
    }
    q = None if query is None else np.ascontiguousarray(query, dtype=np.float32)
    status = ref().ref_codec_head(
        _ptr(dense, _f32p), keys, values, _ptr(q, _f32p),
        _ptr(out["codes"], _i8p), _ptr(out["smoothing"], _f32p),
        _ptr(out["scales"], _f32p), _ptr(out["compensator_keys"], _f32p),
        _ptr(out["compensator_values"], _f32p), _ptr(out["dense_state"], _f32p),
        _ptr(out["projection"], _f32p) if q is not None else _ptr(None, _f32p))
    if status != 0:
        raise ValueError("reference codec rejected the input")
    if q is None:
        del out["projection"]
    return out


# --------------------------------------------------------------------------
# The reference's own quant-only stage (ref_quant_shim.cpp: QuantizeBoundary,
# DequantizeBoundary and ReadWindowState of capsule.cpp at compensator rank 0).
# Capsule layout only: the reference has no provider-layout CPU path.

REF_QUANT_LIB_PATH = ORACLE_DIR / "_ref" / "libgdn_ref_quant.so"
_ref_quant = None


def ref_quant_available() -> bool:
    return REF_QUANT_LIB_PATH.is_file()


def ref_quant() -> ctypes.CDLL:
    global _ref_quant
    if _ref_quant is None:
        if not REF_QUANT_LIB_PATH.is_file():
            raise RuntimeError(f"reference quant-only library not built: {REF_QUANT_LIB_PATH}")
        handle = ctypes.CDLL(str(REF_QUANT_LIB_PATH))
        u64, u32, c_int = ctypes.c_uint64, ctypes.c_uint32, ctypes.c_int
        handle.ref_quant_only_encode.argtypes = [
            _f32p, u64, u32, u32, c_int, _i8p, _f32p, _f32p]
        handle.ref_quant_only_decode.argtypes = [
            _i8p, _f32p, _f32p, u64, u32, u32, c_int, _f32p]
        handle.ref_quant_only_project.argtypes = [
            _i8p, _f32p, _f32p, _f32p, u64, u32, u32, c_int, _f32p]
        for name in ("ref_quant_only_encode", "ref_quant_only_decode",
                     "ref_quant_only_project"):
            getattr(handle, name).restype = c_int
        _ref_quant = handle
    return _ref_quant


def ref_quant_encode(state: np.ndarray, threads: int = 1):
    """Reference quant-only encode of capsule heads: (codes, smoothing, scales)."""
    state = np.ascontiguousarray(state, dtype=np.float32)
    heads, keys, values = state.shape
    codes = np.empty(state.shape, np.int8)
    c = np.empty((heads, keys), np.float32)
    b = np.empty((heads, values), np.float32)
    status = ref_quant().ref_quant_only_encode(
        _ptr(state, _f32p), heads, keys, values, threads, _ptr(codes, _i8p), _ptr(c, _f32p),
        _ptr(b, _f32p))
    if status != 0:
        raise ValueError("reference quantizer rejected the input")
    return codes, c, b


def ref_quant_decode(codes, c, b, threads: int = 1) -> np.ndarray:
    codes = np.ascontiguousarray(codes, dtype=np.int8)
    c = np.ascontiguousarray(c, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    heads, keys, values = codes.shape
    dense = np.empty(codes.shape, np.float32)
    status = ref_quant().ref_quant_only_decode(
        _ptr(codes, _i8p), _ptr(c, _f32p), _ptr(b, _f32p), heads, keys, values, threads,
        _ptr(dense, _f32p))
    if status != 0:
        raise ValueError("reference dequantizer rejected the input")
    return dense


def ref_quant_project(codes, c, b, queries, threads: int = 1) -> np.ndarray:
    codes = np.ascontiguousarray(codes, dtype=np.int8)
    c = np.ascontiguousarray(c, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    q = np.ascontiguousarray(queries, dtype=np.float32)
    heads, keys, values = codes.shape
    out = np.empty((heads, values), np.float32)
    status = ref_quant().ref_quant_only_project(
        _ptr(codes, _i8p), _ptr(c, _f32p), _ptr(b, _f32p), _ptr(q, _f32p), heads, keys, values,
        threads, _ptr(out, _f32p))
    if status != 0:
        raise ValueError("reference readout rejected the input")
    return out


# --------------------------------------------------------------------------
# The reference's capsule wire format (Serialize / Restore, capsule.cpp:446-578).

DEFAULT_GEOMETRY = "a" * 64   # the identity the shim's codec helpers use
CAPSULE_BYTES = 21688          # 128 x 128 head, rank 4, no buffered updates


def _ref_capsule_api() -> ctypes.CDLL:
    handle = ref()
    if not getattr(handle, "_capsule_bound", False):
        u32, u64 = ctypes.c_uint32, ctypes.c_uint64
        handle.ref_serialize_head.argtypes = [_f32p, u32, u32, ctypes.c_char_p, u64, u64,
                                              ctypes.c_void_p, u64]
        handle.ref_serialize_head.restype = u64
        handle.ref_restore_capsule.argtypes = [ctypes.c_void_p, u64, ctypes.c_char_p, u64, u64,
                                               u32, u32, ctypes.c_char_p, u64]
        handle.ref_restore_capsule.restype = ctypes.c_int
        handle._capsule_bound = True
    return handle


def ref_serialize_head(dense: np.ndarray, geometry: str = DEFAULT_GEOMETRY,
                       generation: int = 7, epoch: int = 11) -> bytes:
    """Serialize(FromDenseBoundary(dense)) of the reference library."""
    dense = np.ascontiguousarray(dense, dtype=np.float32)
    keys, values = dense.shape
    out = np.empty(1 << 20, np.uint8)
    size = _ref_capsule_api().ref_serialize_head(
        _ptr(dense, _f32p), keys, values, geometry.encode(), generation, epoch,
        out.ctypes.data, out.size)
    if size == 0:
        raise ValueError("reference rejected the input")
    return out[:size].tobytes()


def ref_restore_capsule(data: bytes, geometry: str = DEFAULT_GEOMETRY, generation: int = 7,
                        epoch: int = 11, keys: int = 128, values: int = 128) -> tuple[bool, str]:
    """Restore() of the reference library: (accepted, rejection message)."""
    buffer = np.frombuffer(data, np.uint8).copy()
    message = ctypes.create_string_buffer(256)
    status = _ref_capsule_api().ref_restore_capsule(
        buffer.ctypes.data, buffer.size, geometry.encode(), generation, epoch, keys, values,
        message, 256)
    return status == 0, message.value.decode()


# --------------------------------------------------------------------------
# Windowed decode path (gdn_window_oracle.c): ReadWindowState / ApplyToken /
# DenseState / QuantizeBoundary of capsule.cpp, with the device ABI's binary16
# record and compensator storage as an option.

WINDOW = 16
QUERY_SCALE = np.float32(0.08838834764831845)  # 128 ** -0.5 as the reference's fp32 constant
_u16p = ctypes.POINTER(ctypes.c_uint16)
_u32p = ctypes.POINTER(ctypes.c_uint32)
_window_ready = False


def _window_lib() -> ctypes.CDLL:
    global _window_ready
    handle = lib()
    if not _window_ready:
        c_int, u32, f32 = ctypes.c_int, ctypes.c_uint32, ctypes.c_float
        handle.oracle_window_read.argtypes = [
            c_int, _i8p, _f32p, _f32p, _f32p, _f32p, u32, _f32p, _f32p, _f32p, _f32p, _f32p]
        handle.oracle_window_step.argtypes = [
            c_int, _i8p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _u32p, f32,
            _f32p, _f32p, _f32p, _f32p, c_int, _f32p]
        handle.oracle_window_dense.argtypes = [
            c_int, _i8p, _f32p, _f32p, _f32p, _f32p, u32, _f32p, _f32p, _f32p, _f32p]
        handle.oracle_quantize_boundary.argtypes = [
            _f32p, u32, c_int, c_int, _i8p, _f32p, _f32p, _f32p, _f32p]
        handle.oracle_quantize_boundary.restype = c_int
        handle.oracle_window_fold.argtypes = [
            c_int, _i8p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _u32p, u32, c_int,
            _i8p, _f32p, _f32p, _f32p, _f32p]
        handle.oracle_window_fold.restype = c_int
        handle.oracle_dense_step.argtypes = [_f32p, f32, _f32p, _f32p, _f32p, _f32p, _f32p]
        handle.oracle_f32_to_f16.argtypes = [f32]
        handle.oracle_f32_to_f16.restype = ctypes.c_uint16
        handle.oracle_f32_to_bf16.argtypes = [f32]
        handle.oracle_f32_to_bf16.restype = ctypes.c_uint16
        _window_ready = True
    return handle


def f32_to_f16_bits(x: float) -> int:
    return int(_window_lib().oracle_f32_to_f16(float(x)))


def f32_to_bf16_bits(x: float) -> int:
    return int(_window_lib().oracle_f32_to_bf16(float(x)))


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_array(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even bfloat16 bits of a finite float32 array."""
    bits = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    return ((bits + 0x7FFF + ((bits >> 16) & 1)) >> 16).astype(np.uint16)


class WindowHead:
    """One head's window: boundary (codes in ``layout``, smoothing, scales,
    optional rank-4 compensators) plus up to 16 records and the position."""

    def __init__(self, codes, smoothing, scales, compensator_keys=None,
                 compensator_values=None, layout: str = "provider"):
        self.provider = 1 if layout == "provider" else 0
        self.codes = np.ascontiguousarray(codes, np.int8).reshape(128, 128)
        self.c = np.ascontiguousarray(smoothing, np.float32).reshape(128)
        self.b = np.ascontiguousarray(scales, np.float32).reshape(128)
        self.ck = None if compensator_keys is None else np.ascontiguousarray(
            compensator_keys, np.float32).reshape(128, RANK)
        self.cv = None if compensator_values is None else np.ascontiguousarray(
            compensator_values, np.float32).reshape(128, RANK)
        self.rdecay = np.zeros(WINDOW, np.float32)
        self.rkeys = np.zeros((WINDOW, 128), np.float32)
        self.rcorr = np.zeros((WINDOW, 128), np.float32)
        self.position = ctypes.c_uint32(0)

    def _boundary(self):
        return (self.provider, _ptr(self.codes, _i8p), _ptr(self.c, _f32p), _ptr(self.b, _f32p),
                _ptr(self.ck, _f32p), _ptr(self.cv, _f32p))

    def read(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        out = np.empty(128, np.float32)
        _window_lib().oracle_window_read(*self._boundary(), self.position.value,
                                         _ptr(self.rdecay, _f32p), _ptr(self.rkeys, _f32p),
                                         _ptr(self.rcorr, _f32p), _ptr(x, _f32p),
                                         _ptr(out, _f32p))
        return out

    def step(self, decay, key, read, query, value, round_storage: bool = True) -> np.ndarray:
        if self.position.value >= WINDOW:
            raise ValueError("window is full")
        arrays = [np.ascontiguousarray(a, np.float32) for a in (key, read, query, value)]
        out = np.empty(128, np.float32)
        _window_lib().oracle_window_step(
            *self._boundary(), _ptr(self.rdecay, _f32p), _ptr(self.rkeys, _f32p),
            _ptr(self.rcorr, _f32p), ctypes.byref(self.position), float(np.float32(decay)),
            *[_ptr(a, _f32p) for a in arrays], int(round_storage), _ptr(out, _f32p))
        return out

    def dense(self) -> np.ndarray:
        out = np.empty((128, 128), np.float32)
        _window_lib().oracle_window_dense(*self._boundary(), self.position.value,
                                          _ptr(self.rdecay, _f32p), _ptr(self.rkeys, _f32p),
                                          _ptr(self.rcorr, _f32p), _ptr(out, _f32p))
        return out

    def fold(self, iterations: int, round_storage: bool = True) -> int:
        """Refit the boundary from the window (records cleared, position 0).
        Compensators are kept (zeros) even for ``iterations == 0``."""
        codes = np.empty_like(self.codes)
        c, b = np.empty_like(self.c), np.empty_like(self.b)
        ck, cv = np.empty((128, RANK), np.float32), np.empty((128, RANK), np.float32)
        status = _window_lib().oracle_window_fold(
            *self._boundary(), _ptr(self.rdecay, _f32p), _ptr(self.rkeys, _f32p),
            _ptr(self.rcorr, _f32p), ctypes.byref(self.position), iterations,
            int(round_storage), _ptr(codes, _i8p), _ptr(c, _f32p), _ptr(b, _f32p),
            _ptr(ck, _f32p), _ptr(cv, _f32p))
        self.codes, self.c, self.b = codes, c, b
        if self.ck is not None or iterations > 0:
            self.ck, self.cv = ck, cv
        return int(status)


def quantize_boundary(dense: np.ndarray, iterations: int = 32, layout: str = "capsule",
                      round_storage: bool = False) -> dict:
    """QuantizeBoundary (capsule.cpp:130-225) of one capsule-order dense head."""
    dense = np.ascontiguousarray(dense, np.float32)
    out = {"codes": np.empty((128, 128), np.int8), "smoothing": np.empty(128, np.float32),
           "scales": np.empty(128, np.float32),
           "compensator_keys": np.empty((128, RANK), np.float32),
           "compensator_values": np.empty((128, RANK), np.float32)}
    status = _window_lib().oracle_quantize_boundary(
        _ptr(dense, _f32p), iterations, 1 if layout == "provider" else 0, int(round_storage),
        _ptr(out["codes"], _i8p), _ptr(out["smoothing"], _f32p), _ptr(out["scales"], _f32p),
        _ptr(out["compensator_keys"], _f32p), _ptr(out["compensator_values"], _f32p))
    out["status"] = int(status)
    return out


def dense_step(state: np.ndarray, decay, key, read, query, value) -> np.ndarray:
    """fp32 GDN step in place on one capsule-order dense head; returns S_new^T query."""
    assert state.dtype == np.float32 and state.flags["C_CONTIGUOUS"]
    arrays = [np.ascontiguousarray(a, np.float32) for a in (key, read, query, value)]
    out = np.empty(128, np.float32)
    _window_lib().oracle_dense_step(_ptr(state, _f32p), float(np.float32(decay)),
                                    *[_ptr(a, _f32p) for a in arrays], _ptr(out, _f32p))
    return out


def qwen_token(decay, beta_bits, key_bits, query_bits, value_bits):
    """The Qwen3.5 decode token of one head as the window step consumes it:
    decay (fp32, exp of the log decay), beta / key / query / value as bf16
    bits.  Returns (decay, key, read, query, value) in fp32: key = beta * k
    (exact), read = decay * k, query = 128^-0.5 * q, value = v."""
    decay = np.float32(decay)
    beta = bf16_bits_to_f32(np.array([beta_bits]))[0]
    k = bf16_bits_to_f32(key_bits)
    q = bf16_bits_to_f32(query_bits)
    v = bf16_bits_to_f32(value_bits)
    return decay, (beta * k).astype(np.float32), (decay * k).astype(np.float32), \
        (QUERY_SCALE * q).astype(np.float32), v.astype(np.float32)


def ref_apply_tokens(dense: np.ndarray, decay, key, read, query, value) -> dict:
    """FromDenseBoundary + ApplyToken of the reference library per token
    (scalar decay broadcast over the keys)."""
    handle = ref()
    if not hasattr(handle, "_apply_ready"):
        u32 = ctypes.c_uint32
        handle.ref_apply_tokens.argtypes = [
            _f32p, u32, u32, u32, _f32p, _f32p, _f32p, _f32p, _f32p, _f32p,
            ctypes.POINTER(ctypes.c_uint8), _f32p, _u32p]
        handle.ref_apply_tokens.restype = ctypes.c_int
        handle._apply_ready = True
    dense = np.ascontiguousarray(dense, np.float32)
    arrays = [np.ascontiguousarray(a, np.float32) for a in (decay, key, read, query, value)]
    tokens = arrays[0].shape[0]
    outputs = np.empty((tokens, 128), np.float32)
    crossed = np.zeros(tokens, np.uint8)
    final = np.empty((128, 128), np.float32)
    position = ctypes.c_uint32(0)
    status = handle.ref_apply_tokens(
        _ptr(dense, _f32p), 128, 128, tokens, *[_ptr(a, _f32p) for a in arrays],
        _ptr(outputs, _f32p), crossed.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8)),
        _ptr(final, _f32p), ctypes.byref(position))
    if status != 0:
        raise ValueError("reference rejected the token sequence")
    return {"outputs": outputs, "crossed": crossed.astype(bool), "dense": final,
            "position": int(position.value)}


def ref_window_read(head: "WindowHead", x: np.ndarray) -> np.ndarray:
    """ReadWindowState of the reference library itself (ref_quant_shim.cpp)
    for a capsule-layout WindowHead at its current position."""
    handle = ref_quant()
    if not hasattr(handle, "_window_ready"):
        u32 = ctypes.c_uint32
        handle.ref_window_read.argtypes = [
            _i8p, _f32p, _f32p, _f32p, _f32p, u32, u32, u32, _f32p, _f32p, _f32p, _f32p, _f32p]
        handle.ref_window_read.restype = ctypes.c_int
        handle._window_ready = True
    if head.provider:
        raise ValueError("the reference reads capsule-layout boundaries")
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(128, np.float32)
    status = handle.ref_window_read(
        _ptr(head.codes, _i8p), _ptr(head.c, _f32p), _ptr(head.b, _f32p), _ptr(head.ck, _f32p),
        _ptr(head.cv, _f32p), 128, 128, head.position.value, _ptr(head.rdecay, _f32p),
        _ptr(head.rkeys, _f32p), _ptr(head.rcorr, _f32p), _ptr(x, _f32p), _ptr(out, _f32p))
    if status != 0:
        raise ValueError("reference window read rejected the input")
    return out


def ref_time_apply_tokens(dense: np.ndarray, decay, key, read, query, value) -> float:
    """Seconds the reference library spends in ApplyToken for these tokens
    (after FromDenseBoundary(dense), which is not timed)."""
    handle = ref()
    if not hasattr(handle, "_time_ready"):
        u32 = ctypes.c_uint32
        handle.ref_time_apply_tokens.argtypes = [
            _f32p, u32, u32, u32, _f32p, _f32p, _f32p, _f32p, _f32p]
        handle.ref_time_apply_tokens.restype = ctypes.c_double
        handle._time_ready = True
    dense = np.ascontiguousarray(dense, np.float32)
    arrays = [np.ascontiguousarray(a, np.float32) for a in (decay, key, read, query, value)]
    seconds = handle.ref_time_apply_tokens(_ptr(dense, _f32p), 128, 128, arrays[0].shape[0],
                                           *[_ptr(a, _f32p) for a in arrays])
    if seconds < 0:
        raise ValueError("reference rejected the token sequence")
    return float(seconds)


def ref_time_capsule(dense: np.ndarray, reps: int) -> tuple[float, float]:
    """(Serialize seconds, Restore seconds) of the reference library for
    `reps` calls each on the capsule of FromDenseBoundary(dense)."""
    handle = ref()
    if not hasattr(handle, "_capsule_time_ready"):
        u32 = ctypes.c_uint32
        dp = ctypes.POINTER(ctypes.c_double)
        handle.ref_time_capsule.argtypes = [_f32p, u32, u32, u32, dp, dp]
        handle.ref_time_capsule.restype = ctypes.c_int
        handle._capsule_time_ready = True
    dense = np.ascontiguousarray(dense, np.float32)
    ser, res = ctypes.c_double(0.0), ctypes.c_double(0.0)
    if handle.ref_time_capsule(_ptr(dense, _f32p), 128, 128, reps, ctypes.byref(ser),
                               ctypes.byref(res)) != 0:
        raise ValueError("reference rejected the head")
    return float(ser.value), float(res.value)
