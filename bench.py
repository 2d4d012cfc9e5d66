"""Benchmark of the B200 GDN state codec hot path.

One step = one pass of the codec over one batch: int8 quantize (fused
smoothing) of every head of the workload, then dequantize of every head
(the batched full-model configuration: 30 GDN layers x 64 request slots x
fp32 state [32, 128, 128] = 61,440 heads, ~4 GB fp32 + 1.07 GB codes,
contiguous slot-major cache, capsule layout).  Under torchrun each rank owns its own 64
slots (weak scaling, no data-path collective); rank r's slots are global slots
64r..64r+63 of the seeded synthetic generator.

Output: one JSON line on rank 0 with the device-timed value (inputs resident
in HBM), an end-to-end value through the public API with host buffers (H2D of
the states and D2H of the reconstruction inside the timed region), the
roofline of the dominant kernel, the CPU baseline, clocks sampled during the
timed region and the launch count.  ``--impl reference`` times the
reference's own CPU codec (its quant-only stage compiled from the reference
sources into oracle/_ref, or the C restatement in oracle/ where that library
is absent) on all host cores instead.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "gdn-state-codec_b200"))
sys.path.insert(0, str(ROOT / "oracle"))  # CPU-baseline leg only (the checker)

METRIC = "codec HBM GB/s (% of B200 peak) and states/sec at 1/2/4/8 B200"
UNIT = "states/s"
# CPU baselines are timed on rank 0 of the one-GPU run only (the host cores are
# shared by every rank of a multi-GPU run).
CPU_AT_N1 = "timed by the one-GPU run only"
SLOTS, LAYERS, HEADS = 64, 30, 32
BYTES_PER_HEAD = {  # algorithmic bytes per head (one launch of each kernel)
    "quantize": 65536 + 16384 + 512 + 512,
    "dequantize": 16384 + 512 + 512 + 65536,
    "projection": 16384 + 512 + 512 + 256 + 512,
}
FALLBACK_HBM_GBS = 6650.0


def parse_args():
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=200)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--impl", choices=["b200", "reference"], default="b200")
    parser.add_argument("--layout", choices=["capsule", "provider"], default="capsule")
    parser.add_argument("--slots", type=int, default=SLOTS,
                        help="request slots per GPU (default: config 2's 64)")
    parser.add_argument("--profile", action="store_true",
                        help="device-resident steps only (for ncu captures of a small case)")
    parser.add_argument("--profile-decode", action="store_true",
                        help="device-resident decode windows only (16 steps + refit per "
                             "window), for ncu captures of the window kernels")
    parser.add_argument("--profile-capsule", action="store_true",
                        help="device-resident capsule serialize + restore only, for ncu "
                             "captures of the capsule kernels")
    parser.add_argument("--profile-full", action="store_true",
                        help="device-resident full-codec launches only (fit + quantize), "
                             "warm-up + steps of them, for ncu captures of the fit kernel")
    return parser.parse_args()


def measured_peak() -> tuple[float, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    try:
        peaks = json.loads(path.read_text())
        return float(peaks["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback"


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons while running."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.proc = None
        self.lines: list[tuple[float, str]] = []   # (host monotonic time, csv line)
        self.thread = None
        self.ready = threading.Event()

    def start(self) -> None:
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu_index}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self) -> None:
        for line in self.proc.stdout:
            self.lines.append((time.monotonic(), line.strip()))
            self.ready.set()

    def wait_ready(self, timeout_s: float = 20.0) -> None:
        """Block until nvidia-smi emits its first sample (NVML start-up takes
        longer on an 8-GPU box than a short timed region lasts)."""
        if self.proc is not None:
            self.ready.wait(timeout_s)

    def stop(self, t0: float | None = None, t1: float | None = None) -> dict:
        """Summarise the samples taken between host times t0 and t1 (the
        timed region).  A region shorter than the sampling interval may hold
        none; then the first sample after t0 stands in, and ``window`` says so."""
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        window = "timed region"
        if t0 is not None:
            deadline = time.monotonic() + 1.0
            while not any(t >= t0 for t, _ in self.lines) and time.monotonic() < deadline:
                time.sleep(0.02)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=5)
        lines = [line for t, line in self.lines
                 if (t0 is None or t >= t0) and (t1 is None or t <= t1)]
        if not lines and t0 is not None:
            lines = [line for t, line in self.lines if t >= t0][:1]
            window = "first sample after the timed region began (region shorter than 100 ms)"
        sm, sm_max, power, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                sm_max.append(float(parts[2]))
                power.append(float(parts[3]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": max(sm_max) if sm_max else None,
            "power_w_max": max(power) if power else None,
            "samples": len(sm),
            "window": window,
            "reasons": sorted(reasons),
        }


def cpu_codec(layout: str, cores: int):
    """The CPU implementation timed beside the GPU: the reference's own
    quant-only stage (QuantizeBoundary / DequantizeBoundary of capsule.cpp at
    compensator rank 0, compiled from the reference sources into
    oracle/_ref/libgdn_ref_quant.so) when it was built, for the capsule layout
    it implements; otherwise the C restatement (oracle/gdn_codec_oracle.c).
    Returns (kind, name, step) where step(states) runs quantize+dequantize."""
    import oracle as oracle_mod  # noqa: PLC0415 - checker/baseline only, never the GPU path

    if layout == "capsule" and oracle_mod.ref_quant_available():
        def step(states):
            z, c, b = oracle_mod.ref_quant_encode(states, threads=cores)
            oracle_mod.ref_quant_decode(z, c, b, threads=cores)
        return "reference", "oracle/_ref/libgdn_ref_quant.so (reference capsule.cpp)", step

    def step(states):  # noqa: F811
        z, c, b = oracle_mod.quantize(states, layout, threads=cores)
        oracle_mod.dequantize(z, c, b, layout=layout, threads=cores)
    return "port", "oracle/gdn_codec_oracle.c", step


def sample_states(layout: str, heads: int):
    """Seeded host heads of the benchmark distribution (per-head
    log-uniform scale in [1e-3, 1], 1% zeros)."""
    import numpy as np

    rng = np.random.default_rng(0)
    scale = (10.0 ** (-3.0 * rng.random((heads, 1, 1)))).astype(np.float32)
    states = rng.standard_normal((heads, 128, 128), dtype=np.float32) * scale
    states[rng.random(states.shape) < 0.01] = 0.0
    if layout == "provider":
        states = np.ascontiguousarray(states.transpose(0, 2, 1))
    return states


def cpu_baseline(layout: str, target_seconds: float = 3.0) -> dict:
    """The CPU codec on all host cores over a bounded sample (rank 0, N=1)."""
    cores = os.cpu_count() or 1
    sample_heads = 2048
    states = sample_states(layout, sample_heads)
    kind, name, step = cpu_codec(layout, cores)
    step(states)  # warm-up pass, then repeat until the time budget is used
    passes, start = 0, time.perf_counter()
    while True:
        step(states)
        passes += 1
        elapsed = time.perf_counter() - start
        if elapsed >= target_seconds:
            break
    return {
        "value": passes * sample_heads / elapsed,
        "unit": UNIT,
        "cores": cores,
        "kind": kind,
        "sample": (f"{passes} passes of quantize+dequantize over {sample_heads} heads of the "
                   f"benchmark distribution ({layout} layout), {name} on {cores} threads, "
                   f"{elapsed:.2f} s wall"),
    }


def arm_config(layout: str, world: int, slots: int = SLOTS) -> dict:
    """The workload both arms report (the reference arm times a bounded
    sample of it, described in its cpu_baseline.sample)."""
    heads = slots * LAYERS * HEADS
    name = "config2" if slots == SLOTS else f"config2 shape with {slots} slots"
    return {
        "workload": f"{name}: 30 GDN layers x {slots} slots x fp32 [32,128,128] per GPU, "
                    "quantize (fused smoothing) + dequantize per step",
        "layout": layout, "heads_per_gpu": heads, "global_batch": heads * world,
        "parallelism": f"dp{world} (request slots sharded, no inter-GPU traffic)",
        "l2": "inputs larger than L2 (9.1 GB touched per step vs 126 MB L2)",
    }


def run_reference(args) -> None:
    """--impl reference: the reference's CPU codec path on all host cores,
    each step a bounded sample of the batched workload."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cores = os.cpu_count() or 1
    sample_heads = 4096
    states = sample_states(args.layout, sample_heads)
    kind, name, step = cpu_codec(args.layout, cores)
    for _ in range(max(args.warmup, 0)):
        step(states)
    start = time.perf_counter()
    for _ in range(args.steps):
        step(states)
    elapsed = time.perf_counter() - start
    value = args.steps * sample_heads / elapsed
    sample = (f"each step: quantize+dequantize of {sample_heads} heads of the benchmark "
              f"distribution (a bounded sample of the 61,440 heads per GPU), {name} on "
              f"{cores} threads")
    print(json.dumps({
        "impl": "reference",
        "metric": METRIC, "value": value, "unit": UNIT, "higher_is_better": True,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": elapsed / args.steps * 1e3, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic",
        "config": arm_config(args.layout, args.gpus, args.slots),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": kind,
                         "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def main() -> None:
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
        return
    if args.warmup < 3 and not (args.profile or args.profile_full or args.profile_decode
                                or args.profile_capsule):
        raise SystemExit("--warmup must be >= 3")

    import torch
    import torch.distributed as dist

    from gdn_state_codec import codec, sharding

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        import datetime

        # Host-side plumbing only (barriers, max over ranks, the report): the
        # codec's data path has no cross-GPU traffic, so no NCCL communicator
        # is created.
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))

    def barrier():
        torch.cuda.synchronize(device)
        sharding.barrier()

    def max_over_ranks(value: float) -> float:
        return sharding.max_over_ranks(value)

    shard = sharding.weak_shard(rank, world, args.slots)
    slots = shard.count
    heads = slots * LAYERS * HEADS
    layout = args.layout
    states = codec.synthesize_states(slots, LAYERS, HEADS, layout=layout, seed=0,
                                     slot_base=shard.base, device=device)
    if args.profile_decode:
        decode_measure(codec, torch, device, barrier, max_over_ranks, slots,
                       windows=args.warmup + args.steps, timed=False)
        barrier()
        if rank == 0:
            print(json.dumps({"profile_decode": True, "heads": heads,
                              "windows": args.warmup + args.steps}))
        if world > 1:
            dist.destroy_process_group()
        return
    if args.profile_full:
        for _ in range(args.warmup + args.steps):
            codec.full_encode(states, layout)
        barrier()
        if rank == 0:
            print(json.dumps({"profile_full": True, "heads": heads,
                              "launches": args.warmup + args.steps}))
        if world > 1:
            dist.destroy_process_group()
        return
    encoded = codec.empty_encoded((slots, LAYERS, HEADS), layout, device)
    dense = torch.empty_like(states)
    stream = torch.cuda.current_stream(device)

    def step(events=None):
        if events is not None:
            events[0].record(stream)
        codec.quantize(states, layout, out=encoded)
        if events is not None:
            events[1].record(stream)
        codec.dequantize(encoded, out=dense)
        if events is not None:
            events[2].record(stream)

    for _ in range(args.warmup):
        step()
    barrier()

    if args.profile_capsule:
        geometry = "0123456789abcdef" * 4
        capsules = torch.empty((heads, codec.CAPSULE_BYTES), dtype=torch.uint8, device=device)
        flat = codec.EncodedStates(encoded.codes.view(-1, 128, 128),
                                   encoded.smoothing.view(-1, 128), encoded.scales.view(-1, 128),
                                   layout)
        for _ in range(args.steps):
            codec.serialize_capsules(flat, geometry=geometry, generation=3, epoch=42,
                                     out=capsules)
            codec.restore_capsules(capsules, layout, geometry=geometry, generation=3, epoch=42)
        barrier()
        if rank == 0:
            print(json.dumps({"profile_capsule": True, "heads": heads, "steps": args.steps}))
        if world > 1:
            dist.destroy_process_group()
        return

    if args.profile:
        queries = codec.synthesize_queries(slots, LAYERS, HEADS, seed=1, device=device)
        outputs = torch.empty(queries.shape, dtype=torch.float32, device=device)
        for _ in range(args.steps):
            step()
            codec.encoded_projection(encoded, queries, out=outputs)
        barrier()
        if rank == 0:
            print(json.dumps({"profile": True, "heads": heads, "steps": args.steps}))
        if world > 1:
            dist.destroy_process_group()
        return

    sampler = ClockSampler(local_rank)
    sampler.start()
    sampler.wait_ready()
    per_step = [[torch.cuda.Event(enable_timing=True) for _ in range(3)]
                for _ in range(args.steps)]
    barrier()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    t0 = time.monotonic()
    start.record(stream)
    for i in range(args.steps):
        step(per_step[i])
    end.record(stream)
    barrier()
    clocks = sampler.stop(t0, time.monotonic())
    elapsed_ms = max_over_ranks(start.elapsed_time(end))
    quant_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in per_step)
    deq_ms = statistics.mean(e[1].elapsed_time(e[2]) for e in per_step)
    ms_per_step = elapsed_ms / args.steps
    value = world * heads * args.steps / (elapsed_ms / 1e3)

    # ---- encoded projection over the same 30-layer cache (config 3 kernel) ----
    queries = codec.synthesize_queries(slots, LAYERS, HEADS, seed=1, slot_base=shard.base,
                                       device=device)
    outputs = torch.empty(queries.shape, dtype=torch.float32, device=device)
    for _ in range(3):
        codec.encoded_projection(encoded, queries, out=outputs)
    barrier()
    p_start = torch.cuda.Event(enable_timing=True)
    p_end = torch.cuda.Event(enable_timing=True)
    proj_iters = max(10, args.steps)
    p_start.record(stream)
    for _ in range(proj_iters):
        codec.encoded_projection(encoded, queries, out=outputs)
    p_end.record(stream)
    barrier()
    proj_ms = max_over_ranks(p_start.elapsed_time(p_end)) / proj_iters

    # ---- full codec (rank-4 fit + int8 stage) on a smaller batch --------------
    full = full_codec_measure(codec, torch, layout, device, barrier, max_over_ranks, rank, world)

    # ---- capsule wire format of the step's encodings ---------------------------
    capsule = capsule_measure(codec, torch, encoded, heads, device, barrier, max_over_ranks,
                              rank, world)

    # ---- end to end through the public API with host buffers -----------------
    e2e = e2e_measure(codec, torch, states, layout, slots, heads, args, device, barrier,
                      max_over_ranks, world)

    # ---- configs 4 and 5 on their own caches (the config-2 buffers freed) ----
    del states, dense, encoded, queries, outputs
    torch.cuda.empty_cache()
    ragged = ragged_measure(codec, torch, layout, device, barrier, rank, world)
    torch.cuda.empty_cache()
    box = box_measure(codec, torch, sharding, layout, device, barrier, max_over_ranks,
                      rank, world)
    torch.cuda.empty_cache()
    decode = decode_measure(codec, torch, device, barrier, max_over_ranks, SLOTS, world=world,
                            rank=rank)
    torch.cuda.empty_cache()

    if rank == 0:
        peak, peak_kind = measured_peak()
        dominant = "quantize" if quant_ms >= deq_ms else "dequantize"
        dom_ms = max(quant_ms, deq_ms)
        achieved = BYTES_PER_HEAD[dominant] * heads / (dom_ms / 1e3) / 1e9
        traffic = committed_traffic(dominant, heads)
        step_gbs = (BYTES_PER_HEAD["quantize"] + BYTES_PER_HEAD["dequantize"]) * heads / (
            ms_per_step / 1e3) / 1e9
        result = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic (seeded on device: N(0,1) x 10^(-3u) per head, "
                                    "1% zeros)",
            "config": arm_config(layout, world, slots),
            "hbm_gbs_per_gpu": step_gbs,
            "hbm_frac_per_gpu": step_gbs / peak,
            "kernels": {
                name: {"ms": ms, "gbs": BYTES_PER_HEAD[name] * heads / (ms / 1e3) / 1e9,
                       "frac": BYTES_PER_HEAD[name] * heads / (ms / 1e3) / 1e9 / peak,
                       "states_per_s": heads / (ms / 1e3)}
                for name, ms in (("quantize", quant_ms), ("dequantize", deq_ms),
                                 ("projection", proj_ms))
            },
            "roofline": {
                "bound": "hbm", "kernel": dominant, "achieved": achieved, "peak": peak,
                "peak_kind": f"{peak_kind} (hbm_gbs, burst copy)", "unit": "GB/s",
                "frac": achieved / peak, "traffic": traffic,
                "bytes_per_head": BYTES_PER_HEAD[dominant], "heads_per_launch": heads,
            },
            "e2e": e2e,
            "full_codec": full,
            "capsule_format": capsule,
            "config4_ragged": ragged,
            "config5_box": box,
            "decode_window": decode,
            "gpu_launches": 2 * args.steps,
            "clocks": clocks,
        }
        result["cpu_baseline"] = (cpu_baseline(layout) if world == 1 else
                                  {"value": None, "unit": UNIT, "skipped": CPU_AT_N1})
        print(json.dumps(result), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def _fits(torch, device, need_bytes: int) -> str | None:
    """None when ``need_bytes`` (plus 2 GiB of headroom) are free on the device,
    else the reason a leg is skipped."""
    free, _ = torch.cuda.mem_get_info(device)
    if free >= need_bytes + (2 << 30):
        return None
    return f"needs {need_bytes / 1e9:.1f} GB, {free / 1e9:.1f} GB free"


def _timed(torch, stream, fn, iters: int):
    """Mean device ms of ``fn`` over ``iters`` launches (CUDA events on the
    launching stream)."""
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(iters):
        fn()
    end.record(stream)
    end.synchronize()
    return start.elapsed_time(end) / iters


def ragged_measure(codec, torch, layout, device, barrier, rank, world):
    """Config 4: a 1,024-slot cache x 30 layers x 32 heads (983,040 heads,
    64 GB fp32 + 17 GB encoded) of which 256 slots, drawn by a seeded
    permutation of 0..1023 (int32, non-contiguous), are quantized, dequantized
    back into the cache and projected, gathered and scattered by slot id.
    A one-GPU configuration: under torchrun it is reported on rank 0 only."""
    if world > 1:
        return {"skipped": "one-GPU configuration (reported by the N=1 run)"}
    cache_slots, active = 1024, 256
    per_slot = LAYERS * HEADS
    heads = active * per_slot
    need = cache_slots * per_slot * (65536 + 16384 + 1024) + active * per_slot * (256 + 512)
    reason = _fits(torch, device, need)
    if reason:
        return {"skipped": reason}
    states = codec.synthesize_states(cache_slots, LAYERS, HEADS, layout=layout, seed=0,
                                     device=device)
    cache = codec.empty_encoded((cache_slots, LAYERS, HEADS), layout, device)
    generator = torch.Generator().manual_seed(0)
    slot_ids = torch.randperm(cache_slots, generator=generator)[:active].to(
        torch.int32).to(device)
    queries = codec.synthesize_queries(active, LAYERS, HEADS, seed=1, device=device)
    outputs = torch.empty(queries.shape, dtype=torch.float32, device=device)
    stream = torch.cuda.current_stream(device)
    legs = {
        "quantize": (lambda: codec.quantize_indexed(states, cache, slot_ids, per_slot),
                     BYTES_PER_HEAD["quantize"]),
        "dequantize": (lambda: codec.dequantize_indexed(cache, states, slot_ids, per_slot),
                       BYTES_PER_HEAD["dequantize"]),
        "projection": (lambda: codec.encoded_projection_indexed(cache, queries, slot_ids,
                                                                per_slot, out=outputs),
                       BYTES_PER_HEAD["projection"]),
    }
    for fn, _ in legs.values():
        for _ in range(3):
            fn()
    barrier()
    result = {"cache_slots": cache_slots, "active_slots": active, "heads": heads,
              "slot_ids": "seeded permutation of 0..1023, first 256, int32"}
    for name, (fn, per_head) in legs.items():
        ms = _timed(torch, stream, fn, 20)
        result[name] = {"ms": ms, "states_per_s": heads / (ms / 1e3),
                        "gbs": per_head * heads / (ms / 1e3) / 1e9}
    del states, cache, queries, outputs
    return result


def box_measure(codec, torch, sharding, layout, device, barrier, max_over_ranks, rank, world):
    """Config 5: 2,048 request slots x 30 layers x 32 heads partitioned by slot
    across the ranks (strong scaling, no inter-GPU traffic); one step =
    quantize + encoded projection of every head of the rank's shard.  Each
    rank also times its two kernels, so the report shows which rank's kernel
    time sets the step, and checks a seeded sample of its heads against the
    CPU oracle after the timed region."""
    shard = sharding.strong_shard(rank, world, 2048)
    per_slot = LAYERS * HEADS
    heads = shard.count * per_slot
    need = heads * (65536 + 16384 + 1024 + 256 + 512)
    reason = _fits(torch, device, need)
    skipped = reason is not None
    if world > 1:  # every rank takes the same steps: skip on all if any must
        skipped = max_over_ranks(float(skipped)) > 0
    if skipped:
        return {"skipped": reason or "another rank lacks the memory"}
    states = codec.synthesize_states(shard.count, LAYERS, HEADS, layout=layout, seed=0,
                                     slot_base=shard.base, device=device)
    encoded = codec.empty_encoded((shard.count, LAYERS, HEADS), layout, device)
    queries = codec.synthesize_queries(shard.count, LAYERS, HEADS, seed=1,
                                       slot_base=shard.base, device=device)
    outputs = torch.empty(queries.shape, dtype=torch.float32, device=device)
    stream = torch.cuda.current_stream(device)

    def step(events=None):
        if events is not None:
            events[0].record(stream)
        codec.quantize(states, layout, out=encoded)
        if events is not None:
            events[1].record(stream)
        codec.encoded_projection(encoded, queries, out=outputs)
        if events is not None:
            events[2].record(stream)

    for _ in range(3):
        step()
    barrier()
    iters = 10
    events = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(iters)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for i in range(iters):
        step(events[i])
    end.record(stream)
    end.synchronize()
    own_ms = start.elapsed_time(end) / iters
    quant_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in events)
    proj_ms = statistics.mean(e[1].elapsed_time(e[2]) for e in events)
    ms = max_over_ranks(own_ms)
    per_rank = sharding.gather_over_ranks({"rank": rank, "slots": shard.count,
                                           "ms_per_step": own_ms, "quantize_ms": quant_ms,
                                           "projection_ms": proj_ms})
    barrier()
    sample = box_parity_sample(codec, torch, layout, states, encoded, queries, outputs, rank)
    mismatches = sharding.sum_over_ranks(sample["mismatches"])
    per_head = BYTES_PER_HEAD["quantize"] + BYTES_PER_HEAD["projection"]
    del states, encoded, queries, outputs
    slowest = max(per_rank, key=lambda r: r["ms_per_step"])
    return {"slots": 2048, "slots_per_gpu": shard.count, "heads_per_gpu": heads,
            "scaling": "strong", "steps": iters, "ms_per_step": ms,
            "states_per_s": 2048 * per_slot / (ms / 1e3),
            "hbm_gbs_per_gpu": per_head * heads / (ms / 1e3) / 1e9,
            "per_rank": per_rank,
            "limiter": (f"rank {slowest['rank']}'s own kernels: quantize "
                        f"{slowest['quantize_ms']:.3f} ms + projection "
                        f"{slowest['projection_ms']:.3f} ms of its {slowest['ms_per_step']:.3f} "
                        f"ms step (max over ranks {ms:.3f} ms); no collective in the step"),
            "parity_sampled_heads": sample["heads"] * world, "mismatches": int(mismatches),
            "parity_checker": sample["checker"]}


def box_parity_sample(codec, torch, layout, states, encoded, queries, outputs, rank,
                      count: int = 512) -> dict:
    """Check a seeded sample of the rank's heads (codes, smoothing, scales and
    projection outputs) against the CPU oracle, outside the timed region."""
    import numpy as np

    import oracle  # the checker (oracle/), never the measured path

    total = encoded.codes.numel() // (128 * 128)
    rng = np.random.default_rng(1000 + rank)
    pick = torch.as_tensor(np.sort(rng.choice(total, size=min(count, total), replace=False)),
                           device=states.device)

    def host(t, inner):
        return t.reshape(total, *inner).index_select(0, pick).cpu().numpy()

    z, c, b = (host(encoded.codes, (128, 128)), host(encoded.smoothing, (128,)),
               host(encoded.scales, (128,)))
    o = host(outputs, (128,))
    q = host(queries.float(), (128,))
    wz, wc, wb = oracle.quantize(host(states, (128, 128)), layout, threads=8)
    wo = oracle.project(wz, wc, wb, q, layout=layout, threads=8)
    bad = ~((z == wz).all(axis=(1, 2)) & (c.view(np.uint32) == wc.view(np.uint32)).all(axis=1)
            & (b.view(np.uint32) == wb.view(np.uint32)).all(axis=1)
            & (o.view(np.uint32) == wo.view(np.uint32)).all(axis=1))
    return {"heads": int(pick.numel()), "mismatches": int(bad.sum()),
            "checker": "oracle.quantize + oracle.project (CPU restatement pinned to the "
                       "reference library) on seeded sampled heads, bit for bit"}


# Algorithmic bytes of one decode step per head at window position p
# (provider codes + smoothing + scales, p records read, the appended record,
# the record decay and position, q / k shared by two heads, value, beta, log
# decay, bf16 output).
def decode_step_bytes(position: float) -> float:
    return (16384 + 512 + 512 + position * (256 + 256 + 4) + (256 + 256 + 4 + 4)
            + 256 + 256 + 2 + 4 + 256)


def capsule_measure(codec, torch, encoded, heads, device, barrier, max_over_ranks, rank,
                    world):
    """The capsule wire format (Serialize / Restore, capsule.cpp:446-578) of
    every head the benchmark step encoded (quant-only boundary: zero
    compensator planes): GPU serialize and fail-closed restore rates, and the
    reference library's own Serialize / Restore on the host cores."""
    geometry = "0123456789abcdef" * 4
    flat = codec.EncodedStates(encoded.codes.view(-1, 128, 128), encoded.smoothing.view(-1, 128),
                               encoded.scales.view(-1, 128), encoded.layout)
    capsules = torch.empty((heads, codec.CAPSULE_BYTES), dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)

    def serialize():
        codec.serialize_capsules(flat, geometry=geometry, generation=3, epoch=42, out=capsules)

    def restore():
        return codec.restore_capsules(capsules, encoded.layout, geometry=geometry,
                                      generation=3, epoch=42)

    for _ in range(2):
        serialize()
        restored = restore()
    ok = bool(torch.equal(restored[0].codes, flat.codes)) and int(restored[3].abs().sum()) == 0
    del restored
    barrier()
    iters = 10
    ser_ms = max_over_ranks(_timed(torch, stream, serialize, iters))
    res_ms = max_over_ranks(_timed(torch, stream, restore, iters))
    barrier()
    ser_bytes = 17408 + codec.CAPSULE_BYTES
    res_bytes = codec.CAPSULE_BYTES + 17408 + 4096
    result = {"heads_per_gpu": heads, "capsule_bytes": codec.CAPSULE_BYTES,
              "serialize_ms": ser_ms, "serialize_states_per_s": world * heads / (ser_ms / 1e3),
              "serialize_gbs_per_gpu": ser_bytes * heads / (ser_ms / 1e3) / 1e9,
              "restore_ms": res_ms, "restore_states_per_s": world * heads / (res_ms / 1e3),
              "restore_gbs_per_gpu": res_bytes * heads / (res_ms / 1e3) / 1e9,
              "round_trip_bit_exact": ok}
    result["cpu_reference"] = (capsule_cpu_reference() if world == 1
                               else {"skipped": CPU_AT_N1})
    return result


def capsule_cpu_reference(sample_heads: int = 64, reps: int = 8):
    """Serialize / Restore of the reference library (oracle/_ref) on the host
    cores over a bounded sample; rates are per-thread rates times threads."""
    import concurrent.futures

    import numpy as np
    import oracle as oracle_mod  # noqa: PLC0415 - baseline only

    if not oracle_mod.ref_available():
        return None
    cores = os.cpu_count() or 1
    heads = sample_states("capsule", sample_heads)
    t0 = time.perf_counter()
    with concurrent.futures.ThreadPoolExecutor(max_workers=cores) as pool:
        times = list(pool.map(lambda h: oracle_mod.ref_time_capsule(h, reps), heads))
    ser = sum(t[0] for t in times)
    res = sum(t[1] for t in times)
    calls = sample_heads * reps
    return {"serialize_states_per_s": calls / ser * cores, "restore_states_per_s": calls / res * cores,
            "cores": cores, "kind": "reference",
            "sample": f"{calls} Serialize and {calls} Restore calls ({sample_heads} heads x {reps}) "
                      f"of oracle/_ref/libgdn_ref.so on {cores} threads, "
                      f"{time.perf_counter() - t0:.2f} s wall"}


def decode_cpu_reference(sample_heads: int = 256, tokens: int = 15,
                         target_seconds: float = 0.2):
    """ApplyToken of the reference library (oracle/_ref, native/src) on the
    host cores: `tokens` Qwen3.5-like tokens (positions 0..14, no window
    crossing) per head over a bounded sample of heads, each head's capsule
    made by FromDenseBoundary first (not timed).  The rate is head-steps per
    second of ApplyToken time per thread, times the threads used."""
    import concurrent.futures

    import numpy as np
    import oracle as oracle_mod  # noqa: PLC0415 - baseline only

    if not oracle_mod.ref_available():
        return None
    cores = os.cpu_count() or 1
    rng = np.random.default_rng(11)
    cases = []
    for _ in range(sample_heads):
        dense = (rng.standard_normal((128, 128)) * 10.0 ** (-3.0 * rng.random())).astype(np.float32)
        decay = np.exp(-(0.005 + 0.095 * rng.random(tokens))).astype(np.float32)
        k = rng.standard_normal((tokens, 128)).astype(np.float32)
        k /= np.linalg.norm(k, axis=1, keepdims=True)
        beta = rng.random(tokens).astype(np.float32)
        q = rng.standard_normal((tokens, 128)).astype(np.float32)
        q *= np.float32(128 ** -0.5) / np.linalg.norm(q, axis=1, keepdims=True)
        v = rng.standard_normal((tokens, 128)).astype(np.float32)
        cases.append((dense, decay, (beta[:, None] * k).astype(np.float32),
                      (decay[:, None] * k).astype(np.float32), q, v))
    busy, steps, t0 = 0.0, 0, time.perf_counter()
    with concurrent.futures.ThreadPoolExecutor(max_workers=cores) as pool:
        while True:
            busy += sum(pool.map(lambda c: oracle_mod.ref_time_apply_tokens(*c), cases))
            steps += sample_heads * tokens
            if busy >= target_seconds * cores or time.perf_counter() - t0 > 20.0:
                break
    per_thread = steps / busy
    return {"head_steps_per_s": per_thread * cores, "per_thread_head_steps_per_s": per_thread,
            "cores": cores, "kind": "reference",
            "sample": f"{steps} head-steps ({sample_heads} heads x {tokens} tokens, ApplyToken "
                      f"of oracle/_ref/libgdn_ref.so, fp32 records) on {cores} threads, "
                      f"{time.perf_counter() - t0:.2f} s wall"}


def decode_token_latency(codec, torch, device, stream, tokens: int = 15):
    """The plugin's decode shape: one request, 30 layers x 32 heads, one
    bf16 step launch per layer per token (runtime.py:750-845).  Device time
    per token of the 30 launches issued eagerly through the Python API, and
    replayed from one CUDA graph that holds them."""
    windows, inputs = [], []
    gen = torch.Generator(device=device).manual_seed(21)
    for layer in range(LAYERS):
        states = codec.synthesize_states(1, 1, HEADS, layout="provider", seed=30 + layer,
                                         device=device).reshape(HEADS, 128, 128)
        windows.append(codec.new_window(codec.quantize(states, "provider")))
        kq = torch.randn((2, HEADS // 2, 128), generator=gen, device=device)
        inputs.append((-0.05 * torch.rand(HEADS, generator=gen, device=device),
                       torch.rand(HEADS, generator=gen, device=device).to(torch.bfloat16),
                       (kq[0] / kq[0].norm(dim=-1, keepdim=True)).to(torch.bfloat16),
                       (kq[1] / kq[1].norm(dim=-1, keepdim=True)).to(torch.bfloat16),
                       torch.randn((HEADS, 128), generator=gen, device=device).to(torch.bfloat16),
                       torch.empty((HEADS, 128), dtype=torch.bfloat16, device=device)))

    def token():
        for window, (log_decay, beta, k, q, v, out) in zip(windows, inputs):
            codec.window_step_bf16(window, log_decay, beta, k, q, v, out=out)

    def reset():
        for window in windows:
            window.positions.zero_()

    token()  # warm-up
    reset()
    torch.cuda.synchronize(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(tokens):
        token()
    end.record(stream)
    end.synchronize()
    eager_us = start.elapsed_time(end) / tokens * 1e3
    reset()
    side = torch.cuda.Stream(device)
    side.wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        token()
    stream.wait_stream(side)
    reset()
    torch.cuda.synchronize(device)
    start.record(stream)
    for _ in range(tokens):
        graph.replay()
    end.record(stream)
    end.synchronize()
    graph_us = start.elapsed_time(end) / tokens * 1e3
    del graph
    runtime = plugin_runtime_token(torch, device, stream, tokens)
    return {"layers": LAYERS, "heads_per_layer": HEADS, "tokens": tokens,
            "eager_us_per_token": eager_us, "graph_us_per_token": graph_us,
            "launches_per_token": LAYERS, "plugin_runtime": runtime}


def plugin_runtime_token(torch, device, stream, tokens: int = 15):
    """The plugin runtime's own decode path (gdn_state_codec.runtime, the
    reference's runtime.py:750-845 on CUDA): one GdnStateCodecRuntime per
    layer, one request slot, `step` called per layer per token, eagerly.
    Reports device time per token (CUDA events) and host time per token and
    per step call (wall clock around the 30 calls, after warm-up)."""
    from gdn_state_codec import _native
    from gdn_state_codec import runtime as runtime_mod
    from gdn_state_codec.config import GdnStateCodecExperiment

    experiment = GdnStateCodecExperiment(_native.library_dir(), "replace", "quant_only", 0,
                                         "vector")
    gen = torch.Generator(device=device).manual_seed(23)
    layers = []
    for layer in range(LAYERS):
        rt = runtime_mod.GdnStateCodecRuntime(experiment, f"model.layers.{layer}.linear_attn")
        ssm = torch.randn((2, HEADS, 128, 128), generator=gen, device=device)
        kq = torch.randn((2, HEADS // 2, 128), generator=gen, device=device)
        kq = (kq / kq.norm(dim=-1, keepdim=True)).to(torch.bfloat16)
        inputs = dict(query=kq[0].reshape(1, 1, HEADS // 2, 128).contiguous(),
                      key=kq[1].reshape(1, 1, HEADS // 2, 128).contiguous(),
                      value=torch.randn((1, 1, HEADS, 128), generator=gen,
                                        device=device).to(torch.bfloat16),
                      log_decay=-0.05 * torch.rand((1, 1, HEADS), generator=gen, device=device),
                      beta=torch.rand((1, 1, HEADS), generator=gen,
                                      device=device).to(torch.bfloat16))
        layers.append((rt, ssm, inputs))

    def token():
        for rt, ssm, inputs in layers:
            rt.step(ssm, 1, query_scale=128 ** -0.5, **inputs)

    token()  # slot encode and first step
    torch.cuda.synchronize(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    host = []
    start.record(stream)
    for _ in range(tokens):  # 15 more steps: the window never needs a refit
        t0 = time.perf_counter()
        token()
        host.append(time.perf_counter() - t0)
    end.record(stream)
    end.synchronize()
    device_us = start.elapsed_time(end) / tokens * 1e3
    host_us = statistics.median(host) * 1e6
    return {"device_us_per_token": device_us, "host_us_per_token": host_us,
            "host_us_per_step_call": host_us / LAYERS,
            "path": "gdn_state_codec.runtime.GdnStateCodecRuntime.step per layer, eager"}


def decode_measure(codec, torch, device, barrier, max_over_ranks, slots, windows: int = 4,
                   timed: bool = True, world: int = 1, rank: int = 0):
    """The Qwen3.5 windowed decode on `slots` x 30 layers x 32 heads per GPU
    (provider layout, quant-only boundary, the plugin's default): each window
    is 16 bf16 decode steps over every head then the quant-only boundary
    refit.  Reports per-step and per-refit device time, head-steps/s and the
    step's algorithmic GB/s; and, for comparison, the dense fp32 GDN step
    (fp32_gdn_step_launch_v1) over the same heads.  Rates are whole-job
    (every rank runs its own `slots`; times are the max over ranks)."""
    heads = slots * LAYERS * HEADS
    states = codec.synthesize_states(slots, LAYERS, HEADS, layout="provider", seed=5,
                                     device=device).reshape(heads, 128, 128)
    window = codec.new_window(codec.quantize(states, "provider"))
    gen = torch.Generator(device=device).manual_seed(9)
    steps = 16
    log_decay = -(0.005 + 0.095 * torch.rand((steps, heads), generator=gen, device=device))
    beta = torch.rand((steps, heads), generator=gen, device=device).to(torch.bfloat16)

    def unit(shape):
        x = torch.randn(shape, generator=gen, device=device)
        return (x / x.norm(dim=-1, keepdim=True)).to(torch.bfloat16)

    keys, queries = unit((steps, heads // 2, 128)), unit((steps, heads // 2, 128))
    values = torch.randn((steps, heads, 128), generator=gen, device=device).to(torch.bfloat16)
    out = torch.empty((heads, 128), dtype=torch.bfloat16, device=device)
    workspace = torch.empty((heads, 128, 128), dtype=torch.float32, device=device)
    stream = torch.cuda.current_stream(device)
    events = []

    def run_window(record):
        nonlocal window
        for t in range(steps):
            if record:
                events.append(("step", torch.cuda.Event(enable_timing=True),
                               torch.cuda.Event(enable_timing=True)))
                events[-1][1].record(stream)
            codec.window_step_bf16(window, log_decay[t], beta[t], keys[t], queries[t],
                                   values[t], out=out)
            if record:
                events[-1][2].record(stream)
        if record:
            events.append(("refit", torch.cuda.Event(enable_timing=True),
                           torch.cuda.Event(enable_timing=True)))
            events[-1][1].record(stream)
        window = codec.window_refit(window, 0, workspace=workspace)
        if record:
            events[-1][2].record(stream)

    if not timed:
        for _ in range(windows):
            run_window(False)
        return None
    run_window(False)  # warm-up window
    barrier()
    for _ in range(windows):
        run_window(True)
    barrier()
    step_ms = [s.elapsed_time(e) for kind, s, e in events if kind == "step"]
    refit_ms = [s.elapsed_time(e) for kind, s, e in events if kind == "refit"]
    step = max_over_ranks(sum(step_ms) / len(step_ms))
    refit = max_over_ranks(sum(refit_ms) / len(refit_ms))
    mean_bytes = sum(decode_step_bytes(p) for p in range(steps)) / steps
    by_position = [sum(step_ms[w * steps + p] for w in range(windows)) / windows
                   for p in (0, steps - 1)]
    del workspace, states
    torch.cuda.empty_cache()
    # dense fp32 GDN step over the same heads (capsule layout, in place)
    dense = codec.synthesize_states(slots, LAYERS, HEADS, layout="capsule", seed=5,
                                    device=device).reshape(heads, 128, 128)
    half = torch.float16
    decay = torch.exp(log_decay[0]).contiguous()
    k16 = keys[0].to(half).repeat_interleave(2, dim=0).contiguous()
    q16 = queries[0].to(half).repeat_interleave(2, dim=0).contiguous()
    v16 = values[0].to(half).contiguous()
    dense_out = torch.empty((heads, 128), dtype=torch.float32, device=device)
    for _ in range(2):
        codec.dense_step(dense, decay, k16, k16, q16, v16, out=dense_out)
    barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(steps):
        codec.dense_step(dense, decay, k16, k16, q16, v16, out=dense_out)
    end.record(stream)
    barrier()
    dense_ms = max_over_ranks(start.elapsed_time(end) / steps)
    del dense
    cpu = decode_cpu_reference() if world == 1 else {"skipped": CPU_AT_N1}
    plugin = decode_token_latency(codec, torch, device, stream)
    return {"cpu_reference": cpu, "plugin_shape_token": plugin, "heads_per_gpu": heads, "layout": "provider", "boundary": "quant-only",
            "windows": windows, "step_ms": step, "step_ms_at_position": {"0": by_position[0],
                                                                      "15": by_position[1]},
            "head_steps_per_s": world * heads / (step / 1e3),
            "step_gbs_per_gpu": mean_bytes * heads / (step / 1e3) / 1e9,
            "step_bytes_per_head_mean": mean_bytes, "refit_ms": refit,
            "window_head_steps_per_s": world * heads * steps / ((steps * step + refit) / 1e3),
            "dense_fp32_step_ms": dense_ms,
            "dense_fp32_step_gbs_per_gpu": 2 * 65536 * heads / (dense_ms / 1e3) / 1e9}


def full_codec_measure(codec, torch, layout, device, barrier, max_over_ranks, rank, world=1):
    """The reference's full encode (FromDenseBoundary: rank-4 fit + int8 stage)
    on 8 slots x 30 layers x 32 heads per GPU (whole-job rate), against the
    reference library itself on the host cores (bounded sample) on rank 0."""
    slots = 8
    heads = slots * LAYERS * HEADS
    states = codec.synthesize_states(slots, LAYERS, HEADS, layout=layout, seed=2,
                                     slot_base=rank * slots, device=device)
    for _ in range(2):
        codec.full_encode(states, layout)
    barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    stream = torch.cuda.current_stream(device)
    iters = 3
    start.record(stream)
    for _ in range(iters):
        codec.full_encode(states, layout)
    end.record(stream)
    barrier()
    ms = max_over_ranks(start.elapsed_time(end)) / iters
    result = {"heads_per_gpu": heads, "ms": ms, "states_per_s": world * heads / (ms / 1e3),
              "bit_exact_to": "FromDenseBoundary (tests/test_gpu_full.py)"}
    result["cpu_reference"] = (full_codec_cpu_reference() if world == 1
                               else {"skipped": CPU_AT_N1})
    return result


def full_codec_cpu_reference(sample_heads: int = 512, target_seconds: float = 2.0):
    """FromDenseBoundary of the reference library (oracle/_ref, compiled from
    native/src) on all host cores, repeated over a bounded sample of heads
    for about ``target_seconds``."""
    import concurrent.futures

    import oracle as oracle_mod  # noqa: PLC0415 - baseline only

    if not oracle_mod.ref_available():
        return None
    cores = os.cpu_count() or 1
    states = sample_states("capsule", sample_heads)
    oracle_mod.ref_codec_head(states[0])  # warm-up
    done, t0 = 0, time.perf_counter()
    with concurrent.futures.ThreadPoolExecutor(max_workers=cores) as pool:
        while True:
            list(pool.map(oracle_mod.ref_codec_head, states))
            done += sample_heads
            elapsed = time.perf_counter() - t0
            if elapsed >= target_seconds:
                break
    return {"states_per_s": done / elapsed, "cores": cores, "kind": "reference",
            "sample": f"{done} heads ({sample_heads} distinct), FromDenseBoundary of "
                      f"oracle/_ref/libgdn_ref.so on {cores} threads, {elapsed:.2f} s wall"}


def committed_traffic(kernel: str, heads: int):
    """DRAM bytes per launch scaled from the committed ncu summary
    (profiles/ncu_traffic.json: bytes per head measured on a capture)."""
    path = ROOT / "profiles" / "ncu_traffic.json"
    try:
        per_head = json.loads(path.read_text())[kernel]["dram_bytes_per_head"]
        return per_head * heads
    except (OSError, KeyError, ValueError, TypeError):
        return None


def bind_host_to_gpu(torch, device) -> dict:
    """Run this process on the host CPUs of the GPU's NUMA node (from sysfs),
    so that pinned buffers allocated next are placed on that node by the
    default first-touch policy.  Returns what was done; the caller restores
    the previous CPU set afterwards."""
    props = torch.cuda.get_device_properties(device)
    bus = f"{props.pci_domain_id:04x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
    node_dir = Path("/sys/bus/pci/devices") / bus
    info = {"pci": bus}
    try:
        info["numa_node"] = int((node_dir / "numa_node").read_text())
        cpus = set()
        for part in (node_dir / "local_cpulist").read_text().strip().split(","):
            lo, _, hi = part.partition("-")
            cpus.update(range(int(lo), int(hi or lo) + 1))
        cpus &= os.sched_getaffinity(0)
        if cpus:
            os.sched_setaffinity(0, cpus)
            info["cpus"] = len(cpus)
        else:
            info["cpus"] = "unchanged (no overlap with the allowed CPUs)"
    except (OSError, ValueError) as exc:
        info["unbound"] = f"{type(exc).__name__}: {exc}"
    return info


def e2e_measure(codec, torch, states, layout, slots, heads, args, device, barrier,
                max_over_ranks, world):
    """Host fp32 states -> H2D -> quantize -> dequantize -> D2H fp32, per layer
    chunk, with copies on their own streams so H2D, compute and D2H overlap.
    The pinned buffers are allocated on the GPU's NUMA node.  After the timed
    region: the whole host output is compared with the device path, and each
    rank's copy rates (H2D alone, D2H alone, both at once, all ranks at the
    same time) are measured to name the host limit."""
    from gdn_state_codec import sharding

    saved_cpus = os.sched_getaffinity(0)
    binding = bind_host_to_gpu(torch, device)
    try:
        host_in = torch.empty(states.shape, dtype=torch.float32, pin_memory=True)
        host_in.copy_(states)
        host_out = torch.empty_like(host_in, pin_memory=True)
    finally:
        os.sched_setaffinity(0, saved_cpus)
    chunk_heads = HEADS * slots  # one layer's worth of heads per chunk
    dev_in = torch.empty_like(states)
    dev_out = torch.empty_like(states)
    enc = codec.empty_encoded((slots, LAYERS, HEADS), layout, device)
    flat = lambda t: t.view(-1, 128, 128)  # noqa: E731
    views = [(flat(host_in)[i:i + chunk_heads], flat(dev_in)[i:i + chunk_heads],
              flat(dev_out)[i:i + chunk_heads], flat(host_out)[i:i + chunk_heads],
              i) for i in range(0, heads, chunk_heads)]
    h2d = torch.cuda.Stream(device)
    d2h = torch.cuda.Stream(device)
    compute = torch.cuda.current_stream(device)
    enc_codes = enc.codes.view(-1, 128, 128)
    enc_c = enc.smoothing.view(-1, 128)
    enc_b = enc.scales.view(-1, 128)

    def one_step():
        for hin, din, dout, hout, i in views:
            with torch.cuda.stream(h2d):
                din.copy_(hin, non_blocking=True)
            ready = torch.cuda.Event()
            ready.record(h2d)
            compute.wait_event(ready)
            part = codec.EncodedStates(enc_codes[i:i + chunk_heads], enc_c[i:i + chunk_heads],
                                       enc_b[i:i + chunk_heads], layout)
            codec.quantize(din, layout, out=part)
            codec.dequantize(part, out=dout)
            done = torch.cuda.Event()
            done.record(compute)
            d2h.wait_event(done)
            with torch.cuda.stream(d2h):
                hout.copy_(dout, non_blocking=True)
        # the next step's first H2D may not overwrite inputs still in use
        h2d.wait_stream(d2h)
        h2d.wait_stream(compute)

    steps = max(3, min(args.steps, 10))
    for _ in range(3):
        one_step()
    torch.cuda.synchronize(device)
    barrier()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record(h2d)
    for _ in range(steps):
        one_step()
    d2h.wait_stream(compute)
    end.record(d2h)
    torch.cuda.synchronize(device)
    barrier()
    ms = max_over_ranks(start.elapsed_time(end)) / steps

    # The whole host output against the device path (every head of the step).
    codec.quantize(states, layout, out=enc)
    codec.dequantize(enc, out=dev_out)
    dev_in.copy_(host_out)
    ok = bool(torch.equal(dev_in, dev_out))

    nbytes = states.numel() * 4

    def copy_rate(copies) -> float:
        """GB/s per direction of ``copies`` (stream, fn) run together, all
        ranks at once."""
        torch.cuda.synchronize(device)
        barrier()
        t0 = torch.cuda.Event(enable_timing=True)
        t0.record(compute)
        for stream, _ in copies:
            stream.wait_event(t0)
        for stream, fn in copies:
            with torch.cuda.stream(stream):
                for _ in range(2):
                    fn()
        for stream, _ in copies:
            compute.wait_stream(stream)
        t1 = torch.cuda.Event(enable_timing=True)
        t1.record(compute)
        t1.synchronize()
        return 2 * nbytes / (t0.elapsed_time(t1) / 1e3) / 1e9

    up = (h2d, lambda: dev_in.copy_(host_in, non_blocking=True))
    down = (d2h, lambda: host_out.copy_(dev_out, non_blocking=True))
    rates = {"h2d_gbs": copy_rate([up]), "d2h_gbs": copy_rate([down]),
             "both_gbs_each_way": copy_rate([up, down])}
    per_rank = sharding.gather_over_ranks({"rank": torch.distributed.get_rank()
                                           if world > 1 else 0, **binding, **rates})
    slowest = min(r["both_gbs_each_way"] for r in per_rank)
    copy_ms = nbytes / (slowest * 1e9) * 1e3
    return {"value": world * heads / (ms / 1e3), "unit": UNIT, "ms_per_step": ms,
            "steps": steps, "h2d_bytes_per_step": nbytes, "d2h_bytes_per_step": nbytes,
            "path": "gdn_state_codec.codec.quantize/dequantize (C ABI) per layer chunk, "
                    "pinned host buffers on the GPU's NUMA node, H2D/compute/D2H on "
                    "separate streams",
            "matches_device_path": ok, "matched_heads": heads,
            "copy_rates_per_rank": per_rank,
            "limiter": (f"host copies: a step moves {nbytes / 1e9:.2f} GB each way per rank; "
                        f"with every rank copying both ways at once the slowest rank moves "
                        f"{slowest:.1f} GB/s each way, so the copies alone take {copy_ms:.1f} ms; "
                        f"the step, with its device kernels overlapped, takes {ms:.1f} ms")}


if __name__ == "__main__":
    main()
