"""The reference plugin's launch sequence, replayed on the GPU.

tests/golden/reference_runtime_protocol.json holds the launches that the
reference's own GdnStateCodecRuntime (src/gdn_state_codec/runtime.py with the
three edits of INTEGRATION.md section 2) makes for one slot of 32 heads:
`provider_initialize_launch_v3` from `_encode_quant_only_provider`, 16 calls
of `windowed_gdn_step_bf16_quant_only_launch_v1` from `step`, the window
refit `window_boundary_launch_v1` from `_refit_boundary`, and two more steps
on the swapped boundary buffers; every pointer is named by the buffer the
plugin allocated (shape, dtype and initial contents as the plugin makes
them).  tests/test_reference_plugin.py re-records it from the reference and
checks it is unchanged; this test needs no reference tree.

Here the same launches run through this repository's C ABI on the GPU, with
the plugin's buffers allocated the plugin's way, and every result is compared
with the CPU oracle bit for bit: the initial encoding, all 18 bf16 outputs,
and the refit boundary.
"""

from __future__ import annotations

import ctypes
import json
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
import window_cases as wc
from gdn_state_codec import _native, codec

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")
FIXTURE = Path(__file__).resolve().parent / "golden" / "reference_runtime_protocol.json"
DTYPES = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16,
          "int8": torch.int8, "int32": torch.int32}


def bits(x):
    return np.ascontiguousarray(x, np.float32).view(np.uint32)


def allocate(spec) -> torch.Tensor:
    dtype = DTYPES[spec["dtype"]]
    if spec["init"] == "zeros":
        return torch.zeros(spec["shape"], dtype=dtype, device=DEV)
    if spec["init"] == "ones":
        return torch.ones(spec["shape"], dtype=dtype, device=DEV)
    return torch.empty(spec["shape"], dtype=dtype, device=DEV)


def test_reference_plugin_protocol_replays_bit_exact():
    protocol = json.loads(FIXTURE.read_text())
    heads = protocol["heads"]
    bufs = {name: allocate(spec) for name, spec in protocol["buffers"].items()}
    state = codec.synthesize_states(1, 1, heads, layout="provider", seed=41, device=DEV)
    bufs["provider_state"].copy_(state.reshape(heads, 128, 128))
    tokens = wc.qwen_tokens(heads, protocol["tokens"], seed=43)
    stream = ctypes.c_void_p(torch.cuda.current_stream(DEV).cuda_stream)

    def load_token(t):
        def put(name, array):
            host = torch.from_numpy(np.ascontiguousarray(array))
            if bufs[name].dtype == torch.bfloat16:
                host = host.view(torch.bfloat16)
            bufs[name].copy_(host.reshape(bufs[name].shape))
        put("log_decay", tokens["log_decay"][t])
        put("beta", tokens["beta"][t])
        put("key", tokens["keys"][t])
        put("query", tokens["queries"][t])
        put("value", tokens["values"][t])

    heads_oracle = None
    steps = refits = 0
    for call in protocol["calls"]:
        args = []
        for a in call["args"]:
            if "stream" in a:
                args.append(stream)
            elif "buf" in a:
                args.append(ctypes.c_void_p(bufs[a["buf"]].data_ptr()))
            else:
                args.append(a["u32"])
        fn = call["fn"]
        if fn.endswith("windowed_gdn_step_bf16_quant_only_launch_v1"):
            load_token(call["token"])
        assert _native.call(fn, *args) == 0, fn
        torch.cuda.synchronize(DEV)
        names = [a.get("buf") for a in call["args"]]
        if fn.endswith("provider_initialize_launch_v3"):
            z, c, b = oracle.quantize(bufs["provider_state"].cpu().numpy(), "provider")
            codes, smoothing, scales = (bufs[names[i]] for i in (3, 2, 4))
            assert np.array_equal(codes.cpu().numpy(), z)
            assert np.array_equal(bits(smoothing.cpu().numpy()), bits(c))
            assert np.array_equal(bits(scales.cpu().numpy()), bits(b))
            heads_oracle = [oracle.WindowHead(z[i], c[i], b[i], layout="provider")
                            for i in range(heads)]
        elif fn.endswith("window_boundary_launch_v1"):
            assert call["args"][-1] == {"u32": 0}  # quant_only: no power iterations
            for h in heads_oracle:
                assert h.fold(0, round_storage=True) == 0
            nz, nc, nb = (bufs[names[i]].cpu().numpy() for i in (10, 11, 12))
            for i, h in enumerate(heads_oracle):
                assert np.array_equal(nz[i], h.codes), f"refit head {i} codes"
                assert np.array_equal(bits(nc[i]), bits(h.c)), f"refit head {i} smoothing"
                assert np.array_equal(bits(nb[i]), bits(h.b)), f"refit head {i} scales"
            refits += 1
        else:
            t = call["token"]
            pos = heads_oracle[0].position.value
            alpha = bufs[names[6]][:, pos].cpu().numpy()  # record_decay of this step
            want = [h.step(*oracle.qwen_token(alpha[i], tokens["beta"][t][i],
                                              tokens["keys"][t][i // 2],
                                              tokens["queries"][t][i // 2],
                                              tokens["values"][t][i]), round_storage=True)
                    for i, h in enumerate(heads_oracle)]
            out = bufs[names[15]].reshape(heads, 128).view(torch.int16).cpu().numpy()
            assert np.array_equal(out.view(np.uint16),
                                  oracle.f32_to_bf16_array(np.stack(want))), f"token {t}"
            steps += 1
    assert steps == protocol["tokens"] and refits == protocol["boundary_refits"] == 1
