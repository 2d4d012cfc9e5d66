"""Multi-rank host logic on CPU (gloo, world size 2; no GPU needed).

Slots shard across ranks with no data-path collective.  What has to hold:
the shards partition the slot range, each rank's encoding of its own slots is
bit-identical to the same slots encoded by one process (heads are
independent and inputs are keyed by global slot id), and timings reduce to
the slowest rank.  The per-rank encode here is the CPU checker standing in
for the GPU launch; the sharding, barrier and reduction code is the one
bench.py runs under NCCL.
"""

from __future__ import annotations

import multiprocessing as mp
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

from gdn_state_codec.sharding import strong_shard, weak_shard

ROOT = Path(__file__).resolve().parents[1]
LAYERS, HEADS = 2, 4


def slot_heads(slot: int) -> np.ndarray:
    """Seeded heads of one global slot ([LAYERS * HEADS, 128, 128])."""
    rng = np.random.default_rng(1000 + slot)
    scale = 10.0 ** (-3.0 * rng.random((LAYERS * HEADS, 1, 1)))
    heads = (rng.standard_normal((LAYERS * HEADS, 128, 128)) * scale).astype(np.float32)
    heads[rng.random(heads.shape) < 0.01] = 0.0
    return heads


def encode_slots(base: int, count: int):
    import oracle

    states = np.concatenate([slot_heads(s) for s in range(base, base + count)])
    return oracle.quantize(states, "capsule")


def test_weak_and_strong_shards_partition_the_slots():
    for world in (1, 2, 4, 8):
        shards = [weak_shard(r, world, 64) for r in range(world)]
        assert [s.base for s in shards] == [64 * r for r in range(world)]
        assert all(s.count == 64 for s in shards)
        for total in (2048, 2047, 9):
            if total < world:
                continue
            parts = [strong_shard(r, world, total) for r in range(world)]
            assert parts[0].base == 0 and parts[-1].stop == total
            assert all(a.stop == b.base for a, b in zip(parts, parts[1:]))
            assert max(p.count for p in parts) - min(p.count for p in parts) <= 1
    with pytest.raises(ValueError):
        weak_shard(2, 2, 64)
    with pytest.raises(ValueError):
        strong_shard(0, 4, 3)


def _rank_main(rank: int, world: int, port: int, total_slots: int, queue) -> None:
    for path in (ROOT / "gdn-state-codec_b200", ROOT / "oracle"):
        sys.path.insert(0, str(path))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    import torch
    import torch.distributed as dist

    from gdn_state_codec import sharding

    try:
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        shard = sharding.strong_shard(rank, world, total_slots)
        z, c, b = encode_slots(shard.base, shard.count)
        sharding.barrier()
        slowest = sharding.max_over_ranks(0.5 + rank)
        assert sharding.sum_over_ranks(1 + rank) == world * (world + 1) / 2
        assert sharding.gather_over_ranks({"rank": rank}) == [{"rank": r} for r in range(world)]
        gathered = sharding.gather_over_ranks((shard.base, shard.count, z, c, b))
        assert sharding.world_size() == world
        dist.destroy_process_group()
        queue.put((rank, "ok", slowest, gathered if rank == 0 else None))
    except Exception as exc:  # noqa: BLE001 - reported to the parent
        queue.put((rank, f"error: {exc!r}", None, None))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_rank_gloo_shards_match_one_process():
    world, total_slots = 2, 5
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, total_slots, queue))
             for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            rank, status, slowest, gathered = queue.get(timeout=180)
            results[rank] = (status, slowest, gathered)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert all(results[r][0] == "ok" for r in range(world)), results
    assert all(results[r][1] == 1.5 for r in range(world))  # max over ranks of 0.5 + rank
    gathered = results[0][2]
    bases = [g[0] for g in gathered]
    counts = [g[1] for g in gathered]
    assert bases == [0, 3] and counts == [3, 2]
    z, c, b = encode_slots(0, total_slots)
    np.testing.assert_array_equal(np.concatenate([g[2] for g in gathered]), z)
    assert np.array_equal(np.concatenate([g[3] for g in gathered]).view(np.uint32),
                          c.view(np.uint32))
    assert np.array_equal(np.concatenate([g[4] for g in gathered]).view(np.uint32),
                          b.view(np.uint32))
