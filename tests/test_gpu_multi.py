"""Slots sharded over the box's GPUs, one process per GPU (a host gloo process
group for the barrier and the max over ranks; the data path has no
cross-GPU traffic, so no NCCL communicator is created): each rank
encodes, dequantizes, projects, takes a decode step, runs the full codec and
serializes capsules for its own slots only, and every slot's bytes equal those
of the same slot run on one GPU.  Heads are independent and every input is
keyed by global slot id, so the sharded outputs concatenate to the 1-GPU
outputs.  Needs two or more GPUs; skipped otherwise."""

from __future__ import annotations

import hashlib
import multiprocessing as mp
import os
import socket
import sys
from pathlib import Path

import pytest
import torch

from gdn_state_codec.sharding import strong_shard

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two or more GPUs")]

ROOT = Path(__file__).resolve().parents[1]
SLOTS, LAYERS, HEADS = 11, 2, 32          # 11 slots: ragged shards at any world size
PER_SLOT = LAYERS * HEADS
GEOMETRY = "0123456789abcdef" * 4


def decode_inputs():
    """One Qwen decode token per head of every global slot (CPU, seeded)."""
    gen = torch.Generator().manual_seed(77)
    heads = SLOTS * PER_SLOT
    log_decay = -0.05 * torch.rand(heads, generator=gen)
    beta = torch.rand(heads, generator=gen).to(torch.bfloat16)
    kq = torch.randn((2, heads // 2, 128), generator=gen)
    kq = (kq / kq.norm(dim=-1, keepdim=True)).to(torch.bfloat16)
    values = torch.randn((heads, 128), generator=gen).to(torch.bfloat16)
    return log_decay, beta, kq[0], kq[1], values


def slot_digests(base: int, count: int, device: torch.device) -> list[str]:
    """SHA-256 per global slot of every output the codec produces for it."""
    from gdn_state_codec import codec

    heads = count * PER_SLOT
    lo, hi = base * PER_SLOT, (base + count) * PER_SLOT
    states = codec.synthesize_states(count, LAYERS, HEADS, layout="provider", seed=3,
                                     slot_base=base, device=device)
    enc = codec.quantize(states, "provider")
    dense = codec.dequantize(enc)
    queries = codec.synthesize_queries(count, LAYERS, HEADS, seed=4, slot_base=base,
                                       device=device)
    projection = codec.encoded_projection(enc, queries)
    log_decay, beta, keys, token_queries, values = decode_inputs()
    window = codec.new_window(codec.quantize(states.reshape(heads, 128, 128), "provider"))
    decoded = codec.window_step_bf16(
        window, log_decay[lo:hi].to(device), beta[lo:hi].to(device),
        keys[lo // 2:hi // 2].to(device), token_queries[lo // 2:hi // 2].to(device),
        values[lo:hi].to(device))
    full = codec.full_encode(states, "provider")
    capsules = codec.serialize_capsules(
        full.encoded, geometry=GEOMETRY, generation=1, epoch=1,
        compensator_keys=full.compensator_keys, compensator_values=full.compensator_values)
    outputs = [enc.codes, enc.smoothing, enc.scales, dense, projection, decoded,
               window.record_keys, capsules]
    rows = [t.contiguous().reshape(count, -1).view(torch.uint8).cpu().numpy() for t in outputs]
    return [hashlib.sha256(b"".join(r[s].tobytes() for r in rows)).hexdigest()
            for s in range(count)]


def _rank_main(rank: int, world: int, port: int, queue) -> None:
    for path in (ROOT / "gdn-state-codec_b200", ROOT / "tests"):
        sys.path.insert(0, str(path))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    import torch.distributed as dist

    from gdn_state_codec import sharding

    try:
        device = torch.device("cuda", rank)
        torch.cuda.set_device(device)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        shard = sharding.strong_shard(rank, world, SLOTS)
        digests = slot_digests(shard.base, shard.count, device)
        sharding.barrier()
        slowest = sharding.max_over_ranks(float(rank))
        dist.destroy_process_group()
        queue.put((rank, "ok", shard.base, digests, slowest))
    except Exception as exc:  # noqa: BLE001 - reported to the parent
        queue.put((rank, f"error: {exc!r}", None, None, None))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_sharded_slots_match_one_gpu():
    world = min(torch.cuda.device_count(), 8)
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            rank, status, base, digests, slowest = queue.get(timeout=300)
            results[rank] = (status, base, digests, slowest)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert all(results[r][0] == "ok" for r in range(world)), results
    assert all(results[r][3] == world - 1 for r in range(world))   # max over ranks
    sharded = [d for r in range(world) for d in results[r][2]]
    assert [results[r][1] for r in range(world)] == \
        [strong_shard(r, world, SLOTS).base for r in range(world)]
    assert sharded == slot_digests(0, SLOTS, torch.device("cuda", 0))
