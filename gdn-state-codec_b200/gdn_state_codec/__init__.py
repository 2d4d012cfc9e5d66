# SPDX-License-Identifier: Apache-2.0
"""GDN State Codec, B200 (sm_100a) backend.

A drop-in for the quant-only hot path of vLLM-HUST/gdn-state-codec: int8
quantize / dequantize of gated-delta-net recurrent state and the encoded
projection o = dequant(S)^T q, as hand-written CUDA kernels behind the
reference's C ABI and library names.
"""

from ._version import __version__

__all__ = ["__version__"]
