# SPDX-License-Identifier: Apache-2.0
"""Host adapter installed by the plugin entry point (vLLM on CUDA).

The reference's adapter (src/gdn_state_codec/adapter.py:1-137) waits for
vLLM-Ascend's Qwen3.5 patch, guards the host class, wraps its ``__init__``
to attach a ``GdnStateCodecRuntime`` per layer and replaces ``_forward_core``
with the windowed decode.  On CUDA the host is vLLM's own
``QwenGatedDeltaNetAttention``; this adapter guards it the same way and
attaches the runtime (``layer._gdn_state_codec_runtime``: slot encode,
reconstruction, boundary readout and shadow checks on the B200 kernels).  It
leaves the forward path alone: the windowed decode that would replace it is
not part of this codec backend.
"""

from __future__ import annotations

import functools
import importlib
from typing import Any

_MARKER = "_gdn_state_codec_b200_installed"
_HOST_MODULE = "vllm.model_executor.layers.mamba.gdn.qwen_gdn_linear_attn"
_HOST_CLASS = "QwenGatedDeltaNetAttention"


def _guard_host(host_class: Any) -> None:
    original = getattr(host_class, "__init__", None)
    if original is None or getattr(host_class, "__module__", None) != _HOST_MODULE:
        raise RuntimeError(
            "gdn_state_codec refuses an unsupported or already patched GDN host: "
            f"{getattr(host_class, '__module__', None)}"
        )


def install() -> dict[str, Any]:
    """Attach the codec runtime to every Qwen3.5 GDN layer built afterwards."""
    module = importlib.import_module(_HOST_MODULE)
    host_class = getattr(module, _HOST_CLASS, None)
    if host_class is None:
        raise RuntimeError(f"gdn_state_codec cannot find the host {_HOST_CLASS}")
    if getattr(host_class, _MARKER, False):
        return {"host": host_class.__module__, "mode": "already-installed"}
    _guard_host(host_class)

    from .runtime import GdnStateCodecRuntime, _logger

    original_init = host_class.__init__

    @functools.wraps(original_init)
    def codec_init(self: Any, config: Any, vllm_config: Any, prefix: str = "",
                   *args: Any, **kwargs: Any) -> None:
        original_init(self, config, vllm_config, prefix, *args, **kwargs)
        runtime = GdnStateCodecRuntime.from_vllm_config(vllm_config, prefix)
        self._gdn_state_codec_runtime = runtime
        if runtime is not None:
            experiment = runtime.experiment
            _logger().warning(
                "GDN State Codec active for %s in %s mode with %s initializer, "
                "%s decode backend, and %d boundary iterations",
                prefix, experiment.mode, experiment.initializer,
                experiment.decode_backend, experiment.boundary_power_iterations)

    host_class.__init__ = codec_init
    setattr(host_class, _MARKER, True)
    return {"host": host_class.__module__, "mode": "runtime-attached"}


__all__ = ["install"]
