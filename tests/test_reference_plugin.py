"""The drop-in claim, checked with the reference's own plugin code.

The reference's vLLM plugin modules (src/gdn_state_codec/config.py and
runtime.py) are loaded from the reference source tree with exactly the three
edits INTEGRATION.md section 2 documents, then:

* its loader `_GdnStateCodecLibraries` (runtime.py:48-237) opens this
  repository's lib/ and binds every symbol it looks for, with argument counts
  that match the declarations in include/statecentric/*.h;
* its device gate accepts "cuda" and refuses "npu";
* its runtime, driven through `_slot` -> `_encode_quant_only_provider` and
  18 `step` calls across a window refit with the launches recorded, makes the
  launch sequence committed in tests/golden/reference_runtime_protocol.json,
  which tests/test_gpu_reference_protocol.py replays on the GPU against the
  oracle.

These tests need the reference source tree (GDN_REFERENCE_ROOT, or a
directory `reference` beside this repository) and are skipped without it.
Nothing here needs a GPU: the libraries load without one.
"""

from __future__ import annotations

import json
from pathlib import Path

import pytest

import reference_plugin
from gdn_state_codec import _native
from test_abi import declared_arity

ROOT = Path(__file__).resolve().parents[1]
FIXTURE = Path(__file__).resolve().parent / "golden" / "reference_runtime_protocol.json"

pytestmark = pytest.mark.skipif(reference_plugin.reference_root() is None,
                                reason="reference source tree not present")


@pytest.fixture(scope="module")
def plugin():
    return reference_plugin.load_reference_plugin(reference_plugin.reference_root())


def test_the_edits_are_the_documented_ones():
    section = ROOT.joinpath("INTEGRATION.md").read_text().split("## 2.")[1].split("## 3.")[0]
    for _, before, after in reference_plugin.EDITS:
        for line in (before.splitlines() + after.splitlines()):
            assert line.strip() in section, f"INTEGRATION.md section 2 lacks {line.strip()!r}"


def test_reference_loader_binds_every_symbol(plugin):
    _, runtime = plugin
    libs = runtime._GdnStateCodecLibraries(_native.library_dir())
    arity = declared_arity()
    bound = {
        "window_step": "windowed_gdn_step_launch_v1",
        "window_step_bf16": "windowed_gdn_step_bf16_launch_v1",
        "window_step_bf16_quant_only": "windowed_gdn_step_bf16_quant_only_launch_v1",
        "window_boundary": "window_boundary_launch_v1",
        "provider_smoothing": "provider_smoothing_launch_v2",
        "provider_quantize": "provider_quantize_launch_v2",
        "provider_initialize": "provider_initialize_launch_v3",
    }
    for attr, symbol in bound.items():
        fn = getattr(libs, attr)
        assert fn is not None, f"the reference loader did not bind {attr}"
        name = "statecentric_gdn_state_codec_" + symbol
        assert fn.__name__ == name
        assert len(fn.argtypes) == arity[name], f"{name}: argument count"
    # The Ascend Cube runtimes are optional in the reference loader and have
    # no CUDA counterpart: the loader finds none and the plugin falls back to
    # the entry points above.
    assert libs.window_boundary_cube_finish is None
    assert libs.boundary_runtime_step is None and libs.decode_runtime_step is None
    libs.close()


def test_reference_device_gate_is_cuda(plugin, monkeypatch):
    config, _ = plugin
    monkeypatch.setenv("GDN_STATE_CODEC_LIBRARY_DIR", str(_native.library_dir()))
    args = ([reference_plugin.ARCHITECTURE], "cuda", True, None, 0)
    experiment = config.parse_gdn_state_codec_experiment(reference_plugin.QUANT_ONLY, *args)
    assert experiment.initializer == "quant_only" and experiment.decode_backend == "vector"
    with pytest.raises(ValueError, match="only supports CUDA"):
        config.parse_gdn_state_codec_experiment(reference_plugin.QUANT_ONLY,
                                                [reference_plugin.ARCHITECTURE], "npu", True,
                                                None, 0)


def test_reference_runtime_launch_protocol_matches_the_fixture(plugin):
    config, runtime = plugin
    protocol = reference_plugin.record_protocol(config, runtime, _native.library_dir())
    assert protocol["boundary_refits"] == 1 and protocol["slot_steps_after"] == 2
    assert json.loads(json.dumps(protocol)) == json.loads(FIXTURE.read_text())
