"""Test infrastructure: the reference's own vLLM plugin modules, loaded from
the reference source tree with the three edits INTEGRATION.md section 2
documents, and a recorder of the launches they make.

The reference files are read (never copied) from GDN_REFERENCE_ROOT, else a
directory `reference` beside this repository; the helpers return None where
that tree is absent (as on the GPU box).  Only tests/ and the fixture script
tests/golden/make_reference_protocol.py use this module.

* load_reference_plugin() builds a package from the reference's
  src/gdn_state_codec/config.py and runtime.py after applying EDITS, with
  vllm.config / vllm.logger replaced by small fakes (the plugin only needs the
  VllmConfig name for a type annotation and a logger).
* record_protocol() drives the unmodified plugin logic, GdnStateCodecRuntime
  (runtime.py:239-843), through `_slot` -> `_encode_quant_only_provider` and
  `tokens` calls of `step` across a window refit, with the library symbols
  bound from this repository's lib/ by `_GdnStateCodecLibraries`
  (runtime.py:48-237) and then swapped for recorders.  The result names every
  pointer argument by the buffer the plugin allocated for it, so that a GPU
  test can replay the plugin's exact launch sequence through the C ABI
  without the reference tree (tests/test_gpu_reference_protocol.py).
"""

from __future__ import annotations

import contextlib
import hashlib
import importlib.util
import logging
import os
import sys
import types
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]
PACKAGE = "_reference_gdn_state_codec"

# (file, text before, text after).  The runtime
# substitutions apply to every occurrence (the stream annotation and
# torch.npu.current_stream(), and the three `.npu_stream` handles).
EDITS = (
    ("config.py",
     'if device_type != "npu":\n        raise ValueError("gdn_state_codec only supports Ascend NPU")',
     'if device_type != "cuda":\n        raise ValueError("gdn_state_codec only supports CUDA (B200, sm_100a)")'),
    ("runtime.py", "torch.npu.", "torch.cuda."),
    ("runtime.py", ".npu_stream", ".cuda_stream"),
)

QUANT_ONLY = {"gdn_state_codec": {"initializer": "quant_only", "boundary_power_iterations": 0,
                                  "decode_backend": "vector", "mode": "replace"}}
ARCHITECTURE = "Qwen3_5ForConditionalGeneration"


def reference_root() -> Path | None:
    root = Path(os.environ.get("GDN_REFERENCE_ROOT", REPO.parent / "reference"))
    return root if (root / "src" / "gdn_state_codec" / "runtime.py").is_file() else None


def source_digests(root: Path) -> dict:
    src = root / "src" / "gdn_state_codec"
    return {name: hashlib.sha256((src / name).read_bytes()).hexdigest()
            for name in ("config.py", "runtime.py")}


def patched_sources(root: Path) -> dict[str, str]:
    src = root / "src" / "gdn_state_codec"
    texts = {name: (src / name).read_text() for name in ("config.py", "runtime.py")}
    for name, before, after in EDITS:
        if before not in texts[name]:
            raise AssertionError(f"edit target not found in {name}: {before!r}")
        texts[name] = texts[name].replace(before, after)
    for name, text in texts.items():
        for npu in ("torch.npu", "npu_stream", '"npu"'):
            if npu in text:
                raise AssertionError(f"{name} still uses {npu} after the edits")
    return texts


@contextlib.contextmanager
def _fake_vllm():
    vllm = types.ModuleType("vllm")
    config = types.ModuleType("vllm.config")
    config.VllmConfig = type("VllmConfig", (), {})
    logger = types.ModuleType("vllm.logger")
    logger.init_logger = logging.getLogger
    vllm.config, vllm.logger = config, logger
    saved = {k: sys.modules.get(k) for k in ("vllm", "vllm.config", "vllm.logger")}
    sys.modules.update({"vllm": vllm, "vllm.config": config, "vllm.logger": logger})
    try:
        yield
    finally:
        for k, v in saved.items():
            if v is None:
                sys.modules.pop(k, None)
            else:
                sys.modules[k] = v


def load_reference_plugin(root: Path):
    """(config module, runtime module) of the reference plugin after EDITS."""
    texts = patched_sources(root)
    src = root / "src" / "gdn_state_codec"
    package = types.ModuleType(PACKAGE)
    package.__path__ = []
    sys.modules[PACKAGE] = package
    modules = {}
    with _fake_vllm():
        for name in ("config", "runtime"):
            spec = importlib.util.spec_from_loader(f"{PACKAGE}.{name}", loader=None,
                                                   origin=str(src / f"{name}.py"))
            module = importlib.util.module_from_spec(spec)
            module.__package__ = PACKAGE
            sys.modules[spec.name] = module
            exec(compile(texts[f"{name}.py"], str(src / f"{name}.py"), "exec"), module.__dict__)
            setattr(package, name, module)
            modules[name] = module
    return modules["config"], modules["runtime"]


def _dtype_name(dtype) -> str:
    return str(dtype).replace("torch.", "")


def record_protocol(config, runtime, lib_dir: Path, heads: int = 32, tokens: int = 18) -> dict:
    """Run the reference runtime's slot encode and `tokens` decode steps with
    its launches recorded instead of executed (host tensors, no GPU)."""
    import torch

    saved_env = os.environ.get("GDN_STATE_CODEC_LIBRARY_DIR")
    os.environ["GDN_STATE_CODEC_LIBRARY_DIR"] = str(lib_dir)
    try:
        experiment = config.parse_gdn_state_codec_experiment(
            QUANT_ONLY, [ARCHITECTURE], "cuda", True, None, 0)
    finally:
        if saved_env is None:
            os.environ.pop("GDN_STATE_CODEC_LIBRARY_DIR", None)
        else:
            os.environ["GDN_STATE_CODEC_LIBRARY_DIR"] = saved_env
    rt = runtime.GdnStateCodecRuntime(experiment, "model.layers.0.linear_attn")
    libs = rt._libraries
    calls: list[dict] = []
    token = [0]
    allocated: dict[int, tuple[str, object]] = {}  # data_ptr -> (field, tensor)

    def recorder(symbol: str, argtypes):
        def call(*args):
            calls.append({"fn": symbol, "token": token[0],
                          "args": [(t, a) for t, a in zip(argtypes, args)]})
            return 0
        return call

    for attr in ("provider_initialize", "provider_smoothing", "provider_quantize",
                 "window_step", "window_step_bf16", "window_step_bf16_quant_only",
                 "window_boundary"):
        fn = getattr(libs, attr)
        if fn is not None:
            setattr(libs, attr, recorder(fn.__name__, list(fn.argtypes)))

    original_allocate = runtime.GdnStateCodecRuntime._allocate_slot

    def allocate(*args):
        slot = original_allocate(*args)
        for field in slot.__slots__:
            value = getattr(slot, field)
            if isinstance(value, torch.Tensor):
                allocated[value.data_ptr()] = (field, value)
        return slot

    fake_stream = types.SimpleNamespace(cuda_stream=0x5EED)
    provider_state = torch.zeros((2, heads, 128, 128), dtype=torch.float32)
    inputs = {
        "query": torch.zeros((1, 1, heads // 2, 128), dtype=torch.bfloat16),
        "key": torch.zeros((1, 1, heads // 2, 128), dtype=torch.bfloat16),
        "value": torch.zeros((1, 1, heads, 128), dtype=torch.bfloat16),
        "log_decay": torch.zeros((1, 1, heads), dtype=torch.float32),
        "beta": torch.zeros((1, 1, heads), dtype=torch.bfloat16),
    }
    with contextlib.ExitStack() as stack:
        def patch(obj, name, value):
            old = getattr(obj, name)
            setattr(obj, name, value)
            stack.callback(setattr, obj, name, old)

        # Uninitialised buffers get a sentinel, so that the recorded initial
        # contents ("zeros" / "ones" / "any") do not depend on host memory.
        real_empty, real_empty_like = torch.empty, torch.empty_like
        patch(torch, "empty", lambda *a, **k: real_empty(*a, **k).fill_(7))
        patch(torch, "empty_like", lambda *a, **k: real_empty_like(*a, **k).fill_(7))
        patch(torch.cuda, "current_stream", lambda *a, **k: fake_stream)
        patch(torch.Tensor, "record_stream", lambda self, stream: None)
        patch(runtime.GdnStateCodecRuntime, "_allocate_slot", staticmethod(allocate))
        for t in range(tokens):
            token[0] = t
            rt.step(provider_state, 1, inputs["query"], inputs["key"], inputs["value"],
                    inputs["log_decay"], inputs["beta"], 128 ** -0.5)
    slot = rt._slots[1]

    names: dict[int, str] = {provider_state[1].data_ptr(): "provider_state"}
    names.update({t.data_ptr(): n for n, t in inputs.items()})
    buffers: dict[str, dict] = {}
    for ptr, (field, tensor) in allocated.items():
        names[ptr] = field
    specs = {"provider_state": provider_state[1], **inputs}
    for ptr, (field, tensor) in allocated.items():
        specs[field] = tensor
    protocol_calls = []
    used: set[str] = set()
    for call in calls:
        args = []
        for ctype, value in call["args"]:
            if ctype.__name__ == "c_void_p":
                if value == fake_stream.cuda_stream and not args:
                    args.append({"stream": True})
                    continue
                if value not in names:
                    raise AssertionError(f"{call['fn']}: pointer argument not a plugin buffer")
                args.append({"buf": names[value]})
                used.add(names[value])
            else:
                args.append({"u32": int(value)})
        protocol_calls.append({"fn": call["fn"], "token": call["token"], "args": args})
    for name in sorted(used):
        tensor = specs[name]
        init = "input" if name in inputs or name == "provider_state" else (
            "zeros" if bool((tensor == 0).all()) else
            "ones" if bool((tensor == 1).all()) else "any")
        buffers[name] = {"shape": list(tensor.shape), "dtype": _dtype_name(tensor.dtype),
                         "init": init}
    return {
        "what": "launch protocol of the reference plugin's GdnStateCodecRuntime "
                "(src/gdn_state_codec/runtime.py) with INTEGRATION.md's three edits, "
                "quant_only initializer, vector decode backend",
        "reference_sha256": source_digests(reference_root() or Path(".")) if reference_root() else {},
        "heads": heads, "tokens": tokens, "experiment": QUANT_ONLY["gdn_state_codec"],
        "slot_steps_after": slot.steps, "boundary_refits": rt.boundary_refits,
        "buffers": buffers, "calls": protocol_calls,
    }
