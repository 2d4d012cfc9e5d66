"""CPU tests of the plugin mirror (gdn_state_codec.config / plugin / runtime /
adapter): the reference's activation and configuration contract
(tests/test_plugin_activation.py, tests/test_manifest03_plugin.py of the
reference) with the device gate moved to CUDA, and the runtime's host logic
with the real library files loaded (no GPU needed) and fakes elsewhere."""

from __future__ import annotations

import sys
import types
from pathlib import Path

import pytest
import torch

from gdn_state_codec import _native, adapter, plugin
from gdn_state_codec import runtime as runtime_mod
from gdn_state_codec.config import GdnStateCodecExperiment, parse_gdn_state_codec_experiment

# The manifest's default activation payload (manifests/vllm-hust-extension-v0.3.json:64-70).
DEFAULT_ACTIVATION = {
    "gdn_state_codec": {
        "mode": "shadow",
        "initializer": "quant_only",
        "boundary_power_iterations": 0,
        "decode_backend": "vector",
    }
}


def _parse(additional_config, device_type="cuda", **overrides):
    args = dict(architectures=["Qwen3_5ForConditionalGeneration"], device_type=device_type,
                enforce_eager=True, speculative_method=None, num_speculative_tokens=0)
    args.update(overrides)
    return parse_gdn_state_codec_experiment(additional_config, **args)


def _clear_switches(monkeypatch):
    for name in ("ENABLE", "KILL_SWITCH", "EVIDENCE"):
        monkeypatch.delenv(plugin._var(name), raising=False)


# -- plugin activation ---------------------------------------------------------

def test_discovery_is_inert_by_default(monkeypatch):
    _clear_switches(monkeypatch)
    monkeypatch.setattr(adapter, "install",
                        lambda: (_ for _ in ()).throw(AssertionError("adapter imported")))
    plugin.register()


def test_kill_switch_wins(monkeypatch):
    _clear_switches(monkeypatch)
    monkeypatch.setenv(plugin._var("ENABLE"), "1")
    monkeypatch.setenv(plugin._var("KILL_SWITCH"), "1")
    monkeypatch.setattr(adapter, "install",
                        lambda: (_ for _ in ()).throw(AssertionError("adapter installed")))
    plugin.register()


def test_explicit_enable_installs_and_emits_evidence(monkeypatch, capsys):
    _clear_switches(monkeypatch)
    monkeypatch.setenv(plugin._var("ENABLE"), "1")
    monkeypatch.setenv(plugin._var("EVIDENCE"), "1")
    monkeypatch.setattr(adapter, "install", lambda: {"host": "fake.host", "mode": "runtime-attached"})
    plugin.register()
    error = capsys.readouterr().err
    assert "EVIDENCE installed mechanism=gdn_state_codec host=fake.host" in error
    assert "pid=" in error


def test_runtime_effective_evidence_is_emitted_once(monkeypatch, capsys):
    _clear_switches(monkeypatch)
    monkeypatch.setenv(plugin._var("EVIDENCE"), "1")
    monkeypatch.setattr(plugin, "_runtime_effective_emitted", False)
    plugin.note_runtime_effective()
    plugin.note_runtime_effective()
    assert capsys.readouterr().err.count("runtime_effective mechanism=gdn_state_codec") == 1


# -- configuration -------------------------------------------------------------

def test_default_activation_parses_on_cuda(monkeypatch, tmp_path):
    monkeypatch.setenv("GDN_STATE_CODEC_LIBRARY_DIR", str(tmp_path))
    experiment = _parse(DEFAULT_ACTIVATION)
    assert experiment == GdnStateCodecExperiment(tmp_path, "shadow", "quant_only", 0, "vector")


def test_not_configured_returns_none(monkeypatch, tmp_path):
    monkeypatch.setenv("GDN_STATE_CODEC_LIBRARY_DIR", str(tmp_path))
    assert _parse({}) is None
    assert _parse(None) is None


def test_device_gate_admits_cuda_only(monkeypatch, tmp_path):
    monkeypatch.setenv("GDN_STATE_CODEC_LIBRARY_DIR", str(tmp_path))
    for device in ("npu", "cpu", "xpu"):
        with pytest.raises(ValueError, match="only supports CUDA"):
            _parse(DEFAULT_ACTIVATION, device_type=device)


def test_library_dir_must_be_absolute(monkeypatch):
    monkeypatch.delenv("GDN_STATE_CODEC_LIBRARY_DIR", raising=False)
    with pytest.raises(ValueError, match="GDN_STATE_CODEC_LIBRARY_DIR"):
        _parse(DEFAULT_ACTIVATION)
    monkeypatch.setenv("GDN_STATE_CODEC_LIBRARY_DIR", "relative/lib")
    with pytest.raises(ValueError, match="GDN_STATE_CODEC_LIBRARY_DIR"):
        _parse(DEFAULT_ACTIVATION)


@pytest.mark.parametrize("change, message", [
    ({"mode": "live"}, "mode must be"),
    ({"initializer": "svd"}, "initializer must be"),
    ({"decode_backend": "tensor"}, "decode_backend must be"),
    ({"boundary_power_iterations": 33}, "boundary_power_iterations"),
    ({"boundary_power_iterations": True}, "boundary_power_iterations"),
    ({"initializer": "exact_svd", "boundary_power_iterations": 0}, "boundary_power_iterations"),
])
def test_invalid_values_are_rejected(monkeypatch, tmp_path, change, message):
    monkeypatch.setenv("GDN_STATE_CODEC_LIBRARY_DIR", str(tmp_path))
    config = {"gdn_state_codec": {**DEFAULT_ACTIVATION["gdn_state_codec"], **change}}
    with pytest.raises(ValueError, match=message):
        _parse(config)


def test_key_set_model_eager_and_speculation_gates(monkeypatch, tmp_path):
    monkeypatch.setenv("GDN_STATE_CODEC_LIBRARY_DIR", str(tmp_path))
    with pytest.raises(ValueError, match="must contain exactly"):
        _parse({"gdn_state_codec": {"mode": "shadow"}})
    with pytest.raises(ValueError, match="Qwen3.5"):
        _parse(DEFAULT_ACTIVATION, architectures=["LlamaForCausalLM"])
    with pytest.raises(ValueError, match="enforce_eager"):
        _parse(DEFAULT_ACTIVATION, enforce_eager=False)
    with pytest.raises(ValueError, match="speculative"):
        _parse(DEFAULT_ACTIVATION, speculative_method="eagle", num_speculative_tokens=2)


# -- runtime ---------------------------------------------------------------------

def _experiment(initializer="quant_only", backend="vector", iterations=0):
    return GdnStateCodecExperiment(_native.library_dir(), "shadow", initializer, iterations,
                                   backend)


def test_libraries_load_from_the_library_dir():
    libraries = runtime_mod._GdnStateCodecLibraries(_native.library_dir())
    assert libraries.provider_initialize is not None
    assert libraries.provider_smoothing is not None and libraries.provider_quantize is not None
    assert libraries.provider_dequantize is not None
    assert libraries.provider_encoded_projection is not None
    # the windowed decode entry points, all resolved from the window libraries
    assert libraries.window_step is not None and libraries.window_step_bf16 is not None
    assert libraries.window_step_bf16_quant_only is not None
    assert libraries.window_boundary is not None
    assert libraries.window_step(*([None] * 16), 1) == 1       # null buffers are refused
    assert libraries.window_boundary(*([None] * 16), 1, 0) == 1


def test_missing_library_file_raises(tmp_path):
    with pytest.raises(RuntimeError, match="native dependency is missing"):
        runtime_mod._GdnStateCodecLibraries(tmp_path)


def test_fallback_reasons_and_slot_invalidation():
    reason = runtime_mod.GdnStateCodecRuntime.decode_fallback_reason
    assert reason(num_prefills=0, num_decodes=1, speculative=True) == "speculative decode"
    assert reason(num_prefills=1, num_decodes=1, speculative=False) == "mixed prefill/decode batch"
    assert reason(num_prefills=0, num_decodes=2, speculative=False) == "multi-request decode batch"
    assert reason(num_prefills=0, num_decodes=1, speculative=False, cache_index_count=3) == \
        "multi-request decode batch"
    assert reason(num_prefills=0, num_decodes=1, speculative=False, cache_index_count=1) is None
    rt = runtime_mod.GdnStateCodecRuntime(_experiment(), "model.layers.0.linear_attn")
    rt._slots = {3: object(), 5: object()}
    rt.invalidate((3, 9))
    assert set(rt._slots) == {5}
    rt.fall_back_to_native("mixed prefill/decode batch")
    rt.fall_back_to_native("mixed prefill/decode batch")
    assert rt._slots == {} and rt.native_fallbacks == 2
    assert rt.native_fallback_reasons == {"mixed prefill/decode batch": 2}


def _fake_slot(heads=4):
    return runtime_mod._EncodedSlot(
        residual=torch.zeros((heads, 128, 128), dtype=torch.int8),
        smoothing=torch.ones((heads, 128)), scales=torch.ones((heads, 128)),
        compensator_keys=torch.zeros((heads, 128, 4), dtype=torch.float16),
        compensator_values=torch.zeros((heads, 128, 4), dtype=torch.float16))


def _decode_inputs(heads=4):
    bf = torch.bfloat16
    return dict(query=torch.zeros((1, 1, heads // 2, 128), dtype=bf),
                key=torch.zeros((1, 1, heads // 2, 128), dtype=bf),
                value=torch.zeros((1, 1, heads, 128), dtype=bf),
                log_decay=torch.zeros((1, 1, heads)), beta=torch.zeros((1, 1, heads), dtype=bf),
                query_scale=128 ** -0.5)


def test_step_validates_inputs_then_launches():
    """The Qwen3.5 input contract is checked first, and the Cube backend has
    no counterpart in this backend."""
    rt = runtime_mod.GdnStateCodecRuntime(_experiment(backend="cube"), "layer")
    rt._slots[0] = _fake_slot()
    with pytest.raises(RuntimeError, match="Cube decode backend is unavailable"):
        rt.step(torch.zeros(1), 0, **_decode_inputs())
    rt2 = runtime_mod.GdnStateCodecRuntime(_experiment(), "layer")
    rt2._slots[0] = _fake_slot()
    bad = _decode_inputs()
    bad["query_scale"] = 0.5
    with pytest.raises(RuntimeError, match="query scale is unsupported"):
        rt2.step(torch.zeros(1), 0, **bad)
    bad = _decode_inputs()
    bad["value"] = bad["value"][..., :64]
    with pytest.raises(RuntimeError, match=r"requires \[1,1,H,128\] value"):
        rt2.step(torch.zeros(1), 0, **bad)


def test_slot_carries_window_buffers():
    slot = _fake_slot(heads=6)
    assert slot.record_keys.shape == (6, 16, 128) and slot.record_keys.dtype == torch.float16
    assert slot.record_corrections.shape == (6, 16, 128)
    assert slot.record_decay.shape == (6, 16) and slot.positions.shape == (6, 8)
    assert slot.residual_workspace.shape == (6, 128, 128)
    assert slot.output.shape == (1, 1, 6, 128) and slot.output.dtype == torch.bfloat16
    assert len(slot.kernel_state_pointers()) == 9


def test_slot_index_out_of_range():
    rt = runtime_mod.GdnStateCodecRuntime(_experiment(), "layer")
    with pytest.raises(RuntimeError, match="cache index is out of range"):
        rt._slot(torch.zeros((2, 4, 128, 128)), 5)


def test_observe_shadow_gate():
    rt = runtime_mod.GdnStateCodecRuntime(_experiment(), "layer")
    reference = torch.ones(64)
    assert rt.observe_shadow(reference * (1 + 1e-3), reference) == pytest.approx(1e-3, rel=1e-3)
    with pytest.raises(RuntimeError, match="relative-RMS gate"):
        rt.observe_shadow(reference * 1.5, reference)
    assert rt.shadow_steps == 2 and rt.shadow_max_relative_rms == pytest.approx(0.5)


# -- adapter -----------------------------------------------------------------------

def test_adapter_attaches_the_runtime_to_the_host(monkeypatch, tmp_path):
    module = types.ModuleType(adapter._HOST_MODULE)

    class QwenGatedDeltaNetAttention:
        def __init__(self, config, vllm_config, prefix="", gqa_interleaved_layout=False):
            self.built = (config, prefix, gqa_interleaved_layout)

    QwenGatedDeltaNetAttention.__module__ = adapter._HOST_MODULE
    module.QwenGatedDeltaNetAttention = QwenGatedDeltaNetAttention
    monkeypatch.setitem(sys.modules, adapter._HOST_MODULE, module)
    receipt = adapter.install()
    assert receipt == {"host": adapter._HOST_MODULE, "mode": "runtime-attached"}
    assert adapter.install()["mode"] == "already-installed"

    monkeypatch.setenv("GDN_STATE_CODEC_LIBRARY_DIR", str(Path(_native.library_dir()).resolve()))
    vllm_config = types.SimpleNamespace(
        model_config=types.SimpleNamespace(
            hf_config=types.SimpleNamespace(architectures=["Qwen3_5ForConditionalGeneration"]),
            enforce_eager=True),
        speculative_config=None,
        additional_config=DEFAULT_ACTIVATION,
        device_config=types.SimpleNamespace(device_type="cuda"))
    layer = QwenGatedDeltaNetAttention("cfg", vllm_config, "model.layers.3.linear_attn", True)
    assert layer.built == ("cfg", "model.layers.3.linear_attn", True)
    assert isinstance(layer._gdn_state_codec_runtime, runtime_mod.GdnStateCodecRuntime)
    plain = types.SimpleNamespace(**{**vars(vllm_config), "additional_config": {}})
    assert QwenGatedDeltaNetAttention("cfg", plain, "x")._gdn_state_codec_runtime is None


def test_adapter_refuses_a_foreign_host(monkeypatch):
    module = types.ModuleType(adapter._HOST_MODULE)

    class QwenGatedDeltaNetAttention:
        pass

    QwenGatedDeltaNetAttention.__module__ = "somebody.else"
    module.QwenGatedDeltaNetAttention = QwenGatedDeltaNetAttention
    monkeypatch.setitem(sys.modules, adapter._HOST_MODULE, module)
    with pytest.raises(RuntimeError, match="refuses an unsupported or already patched"):
        adapter.install()


# -- spawned children ----------------------------------------------------------

def test_child_entry_registers_before_the_target(monkeypatch):
    from gdn_state_codec import bootstrap

    calls = []
    monkeypatch.setattr(plugin, "register", lambda: calls.append("register"))
    result = bootstrap.child_entry(lambda *a, **k: calls.append(("target", a, k)) or "done",
                                   1, key=2)
    assert result == "done"
    assert calls == ["register", ("target", (1,), {"key": 2})]


def test_child_entry_runs_in_a_spawned_interpreter(monkeypatch):
    import multiprocessing
    import operator

    from gdn_state_codec import bootstrap

    _clear_switches(monkeypatch)
    with multiprocessing.get_context("spawn").Pool(1) as pool:
        assert pool.apply(bootstrap.child_entry, (operator.add, 2, 3)) == 5
