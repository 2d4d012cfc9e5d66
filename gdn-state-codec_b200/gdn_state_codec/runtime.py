# SPDX-License-Identifier: Apache-2.0
"""Per-layer GDN state codec runtime on CUDA (B200).

Mirrors the reference's src/gdn_state_codec/runtime.py:
  * ``_GdnStateCodecLibraries`` loads the same library files from
    ``experiment.library_dir`` (runtime.py:47-262), raising the same
    ``RuntimeError`` when a required file is missing, and binds the same entry
    points (provider smoothing / quantize / initialize; the windowed step and
    boundary refit), plus the B200 batched dequantize and encoded projection;
  * ``GdnStateCodecRuntime`` keeps the reference's methods and error
    behaviour: ``from_vllm_config``, ``_encode_dense_boundary`` (exact_svd /
    quant_only), ``_encode_quant_only_provider`` (runtime.py:460-523, the
    fused ``provider_initialize_launch_v3`` on the caller's CUDA stream),
    ``reconstruct``, ``invalidate``, ``decode_fallback_reason``,
    ``fall_back_to_native``, ``step`` and ``observe_shadow``.

The windowed p=16 decode (runtime.py:627-845) runs on the CUDA window
kernels: ``step`` launches ``windowed_gdn_step_bf16_launch_v1`` (or its
quant-only form) on the slot's boundary and records, and every 16 tokens
``_refit_boundary`` folds the window into a new boundary with
``window_boundary_launch_v1``.  The Ascend Cube decode / boundary runtimes
have no counterpart, so ``decode_backend: cube`` raises as the reference does
when that backend is unavailable.  ``boundary_readout`` gives the encoded
projection S^T q of a slot's boundary straight from the int8 codes.
"""

from __future__ import annotations

import ctypes
import logging
import sys
from dataclasses import dataclass
from pathlib import Path
from typing import TYPE_CHECKING

import torch

from . import codec
from .config import GdnStateCodecExperiment, parse_gdn_state_codec_experiment

if TYPE_CHECKING:  # pragma: no cover
    from vllm.config import VllmConfig

KEY_DIMENSION = 128
VALUE_DIMENSION = 128
COMPENSATOR_RANK = 4
WINDOW_SIZE = 16
POSITION_STRIDE = 8
SHADOW_RELATIVE_RMS_LIMIT = 2.0e-2


def _logger():
    """vLLM's logger inside a vLLM process, the standard one elsewhere
    (importing vLLM only for logging costs seconds)."""
    if "vllm.logger" in sys.modules:
        return sys.modules["vllm.logger"].init_logger(__name__)
    return logging.getLogger(__name__)


@dataclass(slots=True)
class _EncodedSlot:
    """One request slot's encoded GDN state for one layer (runtime.py:26-45):
    int8 codes in provider order [H, value, key], smoothing per key, scales
    per value, rank-4 compensators (fp16, zero for quant_only), the p=16
    window records and position, the double-buffered next boundary the refit
    writes, its fp32 workspace and the bf16 step output."""

    residual: torch.Tensor
    smoothing: torch.Tensor
    scales: torch.Tensor
    compensator_keys: torch.Tensor
    compensator_values: torch.Tensor
    record_decay: torch.Tensor | None = None
    record_keys: torch.Tensor | None = None
    record_corrections: torch.Tensor | None = None
    positions: torch.Tensor | None = None
    scratch_residual: torch.Tensor | None = None
    scratch_smoothing: torch.Tensor | None = None
    scratch_scales: torch.Tensor | None = None
    scratch_compensator_keys: torch.Tensor | None = None
    scratch_compensator_values: torch.Tensor | None = None
    residual_workspace: torch.Tensor | None = None
    output: torch.Tensor | None = None
    steps: int = 0

    def __post_init__(self) -> None:
        # runtime.py:392-451: window buffers beside the boundary.
        if self.record_keys is not None:
            return
        heads = self.residual.shape[0]
        device = self.residual.device
        self.record_decay = torch.ones((heads, WINDOW_SIZE), dtype=torch.float32, device=device)
        self.record_keys = torch.zeros((heads, WINDOW_SIZE, KEY_DIMENSION), dtype=torch.float16,
                                       device=device)
        self.record_corrections = torch.zeros((heads, WINDOW_SIZE, VALUE_DIMENSION),
                                              dtype=torch.float16, device=device)
        self.positions = torch.zeros((heads, POSITION_STRIDE), dtype=torch.int32, device=device)
        self.scratch_residual = torch.empty_like(self.residual)
        self.scratch_smoothing = torch.empty_like(self.smoothing)
        self.scratch_scales = torch.empty_like(self.scales)
        self.scratch_compensator_keys = torch.empty_like(self.compensator_keys)
        self.scratch_compensator_values = torch.empty_like(self.compensator_values)
        self.residual_workspace = torch.empty(self.residual.shape, dtype=torch.float32,
                                              device=device)
        self.output = torch.empty((1, 1, heads, VALUE_DIMENSION), dtype=torch.bfloat16,
                                  device=device)

    def kernel_state_pointers(self) -> tuple[int, ...]:
        return (self.residual.data_ptr(), self.smoothing.data_ptr(), self.scales.data_ptr(),
                self.compensator_keys.data_ptr(), self.compensator_values.data_ptr(),
                self.record_decay.data_ptr(), self.record_keys.data_ptr(),
                self.record_corrections.data_ptr(), self.positions.data_ptr())


_DEPENDENCIES = (
    "libstatecentric_gdn_state_codec_window_boundary_kernel.so",
    "libstatecentric_gdn_state_codec_bf16_cube_matmul_kernel.so",
    "libstatecentric_gdn_state_codec_int8_cube_matmul_kernel.so",
    "libstatecentric_gdn_state_codec_encoded_projection_kernel.so",
    "libstatecentric_gdn_state_codec_smoothing_kernel.so",
    "libstatecentric_gdn_state_codec_quantize_kernel.so",
)
_PREFIX = "statecentric_gdn_state_codec_"


def _bind(handle: ctypes.CDLL, name: str, argtypes: list, optional: bool = False):
    function = getattr(handle, _PREFIX + name, None)
    if function is None:
        if optional:
            return None
        raise RuntimeError(f"GDN State Codec native symbol is missing: {_PREFIX + name}")
    function.argtypes = argtypes
    function.restype = ctypes.c_int32
    return function


class _GdnStateCodecLibraries:
    def __init__(self, library_dir: Path) -> None:
        # Every library file depends on the core library in the same
        # directory (rpath $ORIGIN): the directory is self-sufficient.
        self._local_dependencies = []
        for dependency_name in _DEPENDENCIES:
            dependency = library_dir / dependency_name
            if not dependency.is_file():
                raise RuntimeError(f"GDN State Codec native dependency is missing: {dependency}")
            self._local_dependencies.append(ctypes.CDLL(str(dependency), mode=ctypes.RTLD_GLOBAL))
        library = library_dir / "libstatecentric_gdn_state_codec_windowed_gdn_step_kernel.so"
        if not library.is_file():
            raise RuntimeError(f"GDN State Codec kernel library is missing: {library}")
        self._window = ctypes.CDLL(str(library))
        vp, u32 = ctypes.c_void_p, ctypes.c_uint32
        self.window_step = _bind(self._window, "windowed_gdn_step_launch_v1", [vp] * 16 + [u32])
        self.window_step_bf16 = _bind(self._window, "windowed_gdn_step_bf16_launch_v1",
                                      [vp] * 16 + [u32], optional=True)
        self.window_step_bf16_quant_only = _bind(
            self._window, "windowed_gdn_step_bf16_quant_only_launch_v1", [vp] * 16 + [u32],
            optional=True)
        boundary_library = library_dir / "libstatecentric_gdn_state_codec_window_boundary_kernel.so"
        if not boundary_library.is_file():
            raise RuntimeError(f"GDN State Codec boundary library is missing: {boundary_library}")
        self._boundary = ctypes.CDLL(str(boundary_library))
        self.window_boundary = _bind(self._boundary, "window_boundary_launch_v1",
                                     [vp] * 16 + [u32, u32])
        self.window_boundary_cube_finish = _bind(
            self._boundary, "window_boundary_cube_finish_launch_v1", [vp] * 16 + [u32],
            optional=True)
        # The Ascend Cube boundary / decode runtimes have no counterpart here.
        self.boundary_runtime_step = None
        self.decode_runtime_step = None

        self.provider_smoothing = None
        smoothing_library = library_dir / "libstatecentric_gdn_state_codec_smoothing_kernel.so"
        if smoothing_library.is_file():
            self._smoothing = ctypes.CDLL(str(smoothing_library))
            self.provider_smoothing = _bind(self._smoothing, "provider_smoothing_launch_v2",
                                            [vp, vp, vp, u32], optional=True)
        self.provider_quantize = None
        quantize_library = library_dir / "libstatecentric_gdn_state_codec_quantize_kernel.so"
        if quantize_library.is_file():
            self._quantize = ctypes.CDLL(str(quantize_library))
            self.provider_quantize = _bind(self._quantize, "provider_quantize_launch_v2",
                                           [vp] * 5 + [u32], optional=True)
        self.provider_initialize = None
        provider_runtime_library = library_dir / "libstatecentric_gdn_state_codec_provider_runtime.so"
        if provider_runtime_library.is_file():
            self._provider_runtime = ctypes.CDLL(str(provider_runtime_library))
            self.provider_initialize = _bind(self._provider_runtime,
                                             "provider_initialize_launch_v3", [vp] * 5 + [u32],
                                             optional=True)
        # B200 batched entry points (same files: each resolves every symbol).
        projection = self._local_dependencies[3]
        self.provider_dequantize = _bind(projection, "provider_dequantize_launch_v2",
                                         [vp] * 7 + [u32], optional=True)
        self.provider_encoded_projection = _bind(
            projection, "provider_encoded_projection_launch_v1", [vp] * 8 + [u32], optional=True)
        self.initialize = _bind(projection, "initialize_launch_v3", [vp] * 5 + [u32],
                                optional=True)

    def decode_handle(self, states: int) -> int | None:
        return None  # no Cube decode runtime in this backend

    def boundary_handle(self, states: int) -> int | None:
        return None  # no Cube boundary runtime in this backend

    def close(self) -> None:
        pass


class GdnStateCodecRuntime:
    """Eager, single-request codec runtime for one Qwen3.5 GDN layer."""

    def __init__(self, experiment: GdnStateCodecExperiment, prefix: str) -> None:
        self.experiment = experiment
        self.prefix = prefix
        self._libraries = _GdnStateCodecLibraries(experiment.library_dir)
        self._slots: dict[int, _EncodedSlot] = {}
        self._execution_stream: torch.cuda.Stream | None = None
        self._input_contract_validated = False
        self.shadow_steps = 0
        self.shadow_max_relative_rms = 0.0
        self.boundary_refits = 0
        self.native_fallbacks = 0
        self.native_fallback_reasons: dict[str, int] = {}

    def __del__(self) -> None:
        libraries = getattr(self, "_libraries", None)
        if libraries is not None:
            libraries.close()

    @staticmethod
    def from_vllm_config(vllm_config: VllmConfig, prefix: str) -> GdnStateCodecRuntime | None:
        model_config = vllm_config.model_config
        hf_config = model_config.hf_config
        architectures = list(getattr(hf_config, "architectures", ()) or ())
        speculative_config = vllm_config.speculative_config
        speculative_method = (getattr(speculative_config, "method", None)
                              if speculative_config is not None else None)
        speculative_tokens = (int(getattr(speculative_config, "num_speculative_tokens", 0))
                              if speculative_config is not None else 0)
        experiment = parse_gdn_state_codec_experiment(
            vllm_config.additional_config,
            architectures,
            vllm_config.device_config.device_type,
            model_config.enforce_eager,
            speculative_method,
            speculative_tokens,
        )
        if experiment is None:
            return None
        return GdnStateCodecRuntime(experiment, prefix)

    # -- encode ---------------------------------------------------------------

    def _stream(self) -> torch.cuda.Stream:
        stream = self._execution_stream
        if stream is None:
            stream = torch.cuda.current_stream()
            self._execution_stream = stream
        return stream

    def _quantize_capsule(self, residual: torch.Tensor) -> codec.EncodedStates:
        """Quant stage of capsule.cpp:190-225 on [H, key, value] fp32 heads."""
        heads = residual.shape[0]
        out = codec.empty_encoded((heads,), "capsule", residual.device)
        launch = self._libraries.initialize
        if launch is None:
            raise RuntimeError("GDN State Codec batched initializer is unavailable")
        status = launch(self._stream().cuda_stream, residual.data_ptr(), out.smoothing.data_ptr(),
                        out.codes.data_ptr(), out.scales.data_ptr(), heads)
        if status != 0:
            raise RuntimeError(f"GDN State Codec initializer launch failed: {status}")
        return out

    def _encode_dense_boundary(self, dense: torch.Tensor,
                               initializer: str = "exact_svd") -> _EncodedSlot:
        """Encode capsule-order [H, key, value] states (runtime.py:336-388).
        exact_svd takes the rank-4 compensators from a device SVD; the int8
        stage is the native quantizer on the residual."""
        if dense.ndim != 3 or dense.shape[-2:] != (KEY_DIMENSION, VALUE_DIMENSION):
            raise RuntimeError("GDN State Codec requires per-head [128,128] recurrent states")
        dense = dense.to(torch.float32).contiguous()
        heads = dense.shape[0]
        if initializer == "exact_svd":
            left_vectors, singular_values, right_vectors_t = torch.linalg.svd(
                dense, full_matrices=False)
            left = (left_vectors[:, :, :COMPENSATOR_RANK] *
                    singular_values[:, None, :COMPENSATOR_RANK])
            right = right_vectors_t[:, :COMPENSATOR_RANK, :].transpose(-2, -1)
            residual = (dense - torch.bmm(left, right.transpose(-2, -1))).contiguous()
        elif initializer == "quant_only":
            left = torch.zeros((heads, KEY_DIMENSION, COMPENSATOR_RANK), dtype=torch.float32,
                               device=dense.device)
            right = torch.zeros((heads, VALUE_DIMENSION, COMPENSATOR_RANK), dtype=torch.float32,
                                device=dense.device)
            residual = dense
        else:
            raise RuntimeError(f"unsupported GdnStateCodec initializer: {initializer}")
        encoded = self._quantize_capsule(residual)
        return _EncodedSlot(
            # Store [value, key] like the provider path (runtime.py:403-406).
            residual=encoded.codes.transpose(-2, -1).contiguous(),
            smoothing=encoded.smoothing,
            scales=encoded.scales,
            compensator_keys=left.to(torch.float16).contiguous(),
            compensator_values=right.to(torch.float16).contiguous(),
        )

    def _encode_quant_only_provider(self, provider_dense: torch.Tensor) -> _EncodedSlot:
        """runtime.py:460-523: the fused native initializer on [H, value, key]."""
        if provider_dense.ndim != 3 or provider_dense.shape[-2:] != (VALUE_DIMENSION,
                                                                     KEY_DIMENSION):
            raise RuntimeError("GDN State Codec requires provider states shaped [H,128,128]")
        if provider_dense.dtype != torch.float32:
            raise RuntimeError("GDN State Codec provider state must be FP32")
        if not provider_dense.is_contiguous():
            raise RuntimeError("GDN State Codec provider state must be contiguous")
        initialize_launch = self._libraries.provider_initialize
        smoothing_launch = self._libraries.provider_smoothing
        quantize_launch = self._libraries.provider_quantize
        if initialize_launch is None and (smoothing_launch is None or quantize_launch is None):
            raise RuntimeError("GDN State Codec batched provider initializer is unavailable")
        heads = provider_dense.shape[0]
        device = provider_dense.device
        residual = torch.empty_like(provider_dense, dtype=torch.int8)
        smoothing = torch.empty((heads, KEY_DIMENSION), dtype=torch.float32, device=device)
        scales = torch.empty((heads, VALUE_DIMENSION), dtype=torch.float32, device=device)
        stream = self._stream()
        if initialize_launch is not None:
            status = initialize_launch(stream.cuda_stream, provider_dense.data_ptr(),
                                       smoothing.data_ptr(), residual.data_ptr(),
                                       scales.data_ptr(), heads)
            if status != 0:
                raise RuntimeError(f"GDN State Codec provider initializer launch failed: {status}")
        else:
            status = smoothing_launch(stream.cuda_stream, provider_dense.data_ptr(),
                                      smoothing.data_ptr(), heads)
            if status != 0:
                raise RuntimeError(f"GDN State Codec provider smoothing launch failed: {status}")
            status = quantize_launch(stream.cuda_stream, provider_dense.data_ptr(),
                                     smoothing.data_ptr(), residual.data_ptr(), scales.data_ptr(),
                                     heads)
            if status != 0:
                raise RuntimeError(f"GDN State Codec provider quantize launch failed: {status}")
        return _EncodedSlot(
            residual=residual,
            smoothing=smoothing,
            scales=scales,
            compensator_keys=torch.zeros((heads, KEY_DIMENSION, COMPENSATOR_RANK),
                                         dtype=torch.float16, device=device),
            compensator_values=torch.zeros((heads, VALUE_DIMENSION, COMPENSATOR_RANK),
                                           dtype=torch.float16, device=device),
        )

    # -- decode-side helpers ----------------------------------------------------

    @staticmethod
    def reconstruct(slot: _EncodedSlot) -> torch.Tensor:
        """Dense [H, key, value] state of a slot (runtime.py:550-561), by the
        native dequantize in the reference's DenseState order
        ((c * z) / 127) * b + sum_r K V (capsule.cpp:229-251)."""
        encoded = codec.EncodedStates(slot.residual, slot.smoothing, slot.scales, "provider")
        dense = codec.dequantize(encoded,
                                 compensator_keys=slot.compensator_keys.to(torch.float32).contiguous(),
                                 compensator_values=slot.compensator_values.to(torch.float32).contiguous())
        return dense.transpose(-2, -1)

    def boundary_readout(self, slot: _EncodedSlot, query: torch.Tensor) -> torch.Tensor:
        """Encoded projection o[h] = S_h^T q_h of the slot's boundary from the
        int8 codes (ReadWindowState's boundary term, capsule.cpp:281-304);
        query bf16 [H, 128], output fp32 [H, 128]."""
        heads = slot.residual.shape[0]
        if query.shape != (heads, KEY_DIMENSION) or query.dtype != torch.bfloat16:
            raise RuntimeError("GDN State Codec boundary readout requires bf16 [H,128] queries")
        launch = self._libraries.provider_encoded_projection
        if launch is None:
            raise RuntimeError("GDN State Codec encoded projection is unavailable")
        query = query.contiguous()
        keys = slot.compensator_keys.to(torch.float32).contiguous()
        values = slot.compensator_values.to(torch.float32).contiguous()
        out = torch.empty((heads, VALUE_DIMENSION), dtype=torch.float32, device=query.device)
        status = launch(self._stream().cuda_stream, slot.residual.data_ptr(),
                        slot.smoothing.data_ptr(), slot.scales.data_ptr(), keys.data_ptr(),
                        values.data_ptr(), query.data_ptr(), out.data_ptr(), heads)
        if status != 0:
            raise RuntimeError(f"GDN State Codec encoded projection launch failed: {status}")
        keys.record_stream(self._stream())
        values.record_stream(self._stream())
        return out

    def invalidate(self, cache_indices: tuple[int, ...]) -> None:
        for cache_index in cache_indices:
            self._slots.pop(cache_index, None)

    @staticmethod
    def decode_fallback_reason(*, num_prefills: int, num_decodes: int, speculative: bool,
                               cache_index_count: int | None = None) -> str | None:
        """Why this invocation must use the native recurrent op (runtime.py:567-584)."""
        if speculative:
            return "speculative decode"
        if num_prefills > 0 and num_decodes > 0:
            return "mixed prefill/decode batch"
        if num_decodes > 0 and (num_decodes != 1 or
                                (cache_index_count is not None and cache_index_count != 1)):
            return "multi-request decode batch"
        return None

    def fall_back_to_native(self, reason: str) -> None:
        """Discard compressed shadows before the provider updates dense state."""
        cleared_slots = len(self._slots)
        self._slots.clear()
        self.native_fallbacks += 1
        count = self.native_fallback_reasons.get(reason, 0) + 1
        self.native_fallback_reasons[reason] = count
        if count == 1:
            _logger().info("GDN State Codec %s uses native fallback for %s "
                           "(%d compressed slots invalidated)", self.prefix, reason, cleared_slots)

    def _slot(self, provider_state: torch.Tensor, cache_index: int) -> _EncodedSlot:
        slot = self._slots.get(cache_index)
        if slot is not None:
            return slot
        if cache_index < 0 or cache_index >= provider_state.shape[0]:
            raise RuntimeError("GDN State Codec cache index is out of range")
        provider_dense = provider_state[cache_index]
        if self.experiment.initializer == "quant_only":
            slot = self._encode_quant_only_provider(provider_dense)
        else:
            dense = provider_dense.transpose(-2, -1).contiguous()
            slot = self._encode_dense_boundary(dense, self.experiment.initializer)
        self._slots[cache_index] = slot
        _logger().info("GDN State Codec initialized %s cache slot %d", self.prefix, cache_index)
        return slot

    def _refit_boundary(self, slot: _EncodedSlot) -> None:
        """Fold the slot's full window into a new boundary (runtime.py:627-733):
        window_boundary_launch_v1 writes the scratch boundary, clears the
        records and resets the position; the buffers then swap."""
        stream = self._stream()
        status = self._libraries.window_boundary(
            stream.cuda_stream, *slot.kernel_state_pointers(), slot.scratch_residual.data_ptr(),
            slot.scratch_smoothing.data_ptr(), slot.scratch_scales.data_ptr(),
            slot.scratch_compensator_keys.data_ptr(), slot.scratch_compensator_values.data_ptr(),
            slot.residual_workspace.data_ptr(), slot.residual.shape[0],
            self.experiment.boundary_power_iterations)
        if status != 0:
            raise RuntimeError(f"GDN State Codec boundary-refit launch failed: {status}")
        # The launch bypasses the allocator's stream tracking: keep the old
        # boundary alive until the refit has read it.
        for tensor in (slot.residual, slot.smoothing, slot.scales, slot.compensator_keys,
                       slot.compensator_values, slot.residual_workspace):
            tensor.record_stream(stream)
        slot.residual, slot.scratch_residual = slot.scratch_residual, slot.residual
        slot.smoothing, slot.scratch_smoothing = slot.scratch_smoothing, slot.smoothing
        slot.scales, slot.scratch_scales = slot.scratch_scales, slot.scales
        slot.compensator_keys, slot.scratch_compensator_keys = (slot.scratch_compensator_keys,
                                                                slot.compensator_keys)
        slot.compensator_values, slot.scratch_compensator_values = (
            slot.scratch_compensator_values, slot.compensator_values)
        slot.steps = 0
        self.boundary_refits += 1
        log = _logger().warning if self.experiment.mode == "shadow" else _logger().info
        log("GDN State Codec boundary %s refits=%d shadow_max_relative_rms=%.8g", self.prefix,
            self.boundary_refits, self.shadow_max_relative_rms)

    def step(self, provider_state: torch.Tensor, cache_index: int, query: torch.Tensor,
             key: torch.Tensor, value: torch.Tensor, log_decay: torch.Tensor,
             beta: torch.Tensor, query_scale: float) -> torch.Tensor:
        """Windowed decode step (runtime.py:750-845): refit at a full window,
        validate the Qwen3.5 input contract once, then one bf16 step launch
        (the quant-only kernel for quant-only boundaries without refit power
        iterations); returns the slot's bf16 output [1, 1, H, 128]."""
        slot = self._slot(provider_state, cache_index)
        if slot.steps == WINDOW_SIZE:
            self._refit_boundary(slot)
        elif slot.steps > WINDOW_SIZE:
            raise RuntimeError("GDN State Codec runtime window position exceeded p=16")
        heads = slot.residual.shape[0]
        if not self._input_contract_validated:
            query_shape = (1, 1, heads // 2, KEY_DIMENSION)
            if query.shape != query_shape or key.shape != query_shape:
                raise RuntimeError("GDN State Codec Qwen3.5 gate requires [1,1,H/2,128] query/key")
            if value.shape != (1, 1, heads, VALUE_DIMENSION):
                raise RuntimeError("GDN State Codec Qwen3.5 gate requires [1,1,H,128] value")
            if log_decay.shape != (1, 1, heads) or beta.shape != (1, 1, heads):
                raise RuntimeError("GDN State Codec Qwen3.5 gate requires [1,1,H] decay/beta")
            if log_decay.dtype != torch.float32:
                raise RuntimeError("GDN State Codec Qwen3.5 gate requires FP32 log decay")
            if query.dtype != torch.bfloat16 or key.dtype != torch.bfloat16:
                raise RuntimeError("GDN State Codec Qwen3.5 gate requires BF16 query/key")
            if value.dtype != torch.bfloat16 or beta.dtype != torch.bfloat16:
                raise RuntimeError("GDN State Codec Qwen3.5 gate requires BF16 value/beta")
            if abs(query_scale - KEY_DIMENSION ** -0.5) > 1.0e-8:
                raise RuntimeError("GDN State Codec Qwen3.5 query scale is unsupported")
            if not all(t.is_contiguous() for t in (query, key, value, log_decay, beta)):
                raise RuntimeError("GDN State Codec Qwen3.5 inputs must be contiguous")
            self._input_contract_validated = True
        vector = self.experiment.decode_backend == "vector"
        if vector:
            vector_step = self._libraries.window_step_bf16
            if (self.experiment.initializer == "quant_only"
                    and self.experiment.boundary_power_iterations == 0
                    and self._libraries.window_step_bf16_quant_only is not None):
                vector_step = self._libraries.window_step_bf16_quant_only
            if vector_step is None:
                raise RuntimeError("GDN State Codec vector decode backend is unavailable")
        else:
            decode_handle = self._libraries.decode_handle(heads)
            if decode_handle is None or self._libraries.decode_runtime_step is None:
                raise RuntimeError("GDN State Codec Cube decode backend is unavailable")
        pointers = (self._stream().cuda_stream, *slot.kernel_state_pointers(),
                    log_decay.data_ptr(), beta.data_ptr(), key.data_ptr(), query.data_ptr(),
                    value.data_ptr(), slot.output.data_ptr())
        if vector:
            status = vector_step(*pointers, heads)
        else:
            status = self._libraries.decode_runtime_step(decode_handle, *pointers, heads)
        if status != 0:
            raise RuntimeError(f"GDN State Codec decode-step launch failed: {status}")
        slot.steps += 1
        return slot.output

    def observe_shadow(self, compressed: torch.Tensor, reference: torch.Tensor) -> float:
        """Relative RMS of a compressed output against the dense path, gated
        at 2e-2 (runtime.py:847-868)."""
        difference = compressed.to(torch.float32) - reference.to(torch.float32)
        denominator = reference.to(torch.float32).square().sum().clamp_min(1.0e-30)
        relative_rms = float(torch.sqrt(difference.square().sum() / denominator).cpu())
        self.shadow_steps += 1
        self.shadow_max_relative_rms = max(self.shadow_max_relative_rms, relative_rms)
        _logger().info("GDN State Codec shadow %s step=%d relative_rms=%.8g max=%.8g",
                       self.prefix, self.shadow_steps, relative_rms, self.shadow_max_relative_rms)
        if relative_rms >= SHADOW_RELATIVE_RMS_LIMIT:
            raise RuntimeError("GDN State Codec shadow output exceeded the relative-RMS gate: "
                               f"{relative_rms:.8g}")
        return relative_rms


__all__ = ["GdnStateCodecRuntime"]
