# SPDX-License-Identifier: Apache-2.0
"""Request-slot sharding across GPUs of one box (one process per GPU).

GDN recurrent state is independent per request slot, so the codec shards by
slot with no data-path collective: rank r owns a contiguous block of global
slot ids and touches only its own HBM.  The only cross-rank operations are
host-side plumbing: a barrier around timed regions, the max over ranks of a
device-measured time and the gathering of per-rank figures for the report.
They run on a host (gloo) process group, on the GPU box as in the CPU tests,
so no NCCL communicator is created at all.
"""

from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class SlotShard:
    """Global slot ids [base, base + count) owned by one rank."""

    rank: int
    world: int
    base: int
    count: int

    @property
    def stop(self) -> int:
        return self.base + self.count


def weak_shard(rank: int, world: int, slots_per_rank: int) -> SlotShard:
    """Fixed work per rank: rank r owns slots [r * n, (r + 1) * n)."""
    _check_rank(rank, world)
    if slots_per_rank < 1:
        raise ValueError("slots_per_rank must be >= 1")
    return SlotShard(rank, world, rank * slots_per_rank, slots_per_rank)


def strong_shard(rank: int, world: int, total_slots: int) -> SlotShard:
    """Fixed total work: contiguous blocks of total_slots / world slots, the
    first total_slots % world ranks taking one extra slot."""
    _check_rank(rank, world)
    if total_slots < world:
        raise ValueError("need at least one slot per rank")
    per, extra = divmod(total_slots, world)
    base = rank * per + min(rank, extra)
    return SlotShard(rank, world, base, per + (1 if rank < extra else 0))


def _check_rank(rank: int, world: int) -> None:
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")


def _distributed():
    import torch.distributed as dist

    return dist if dist.is_available() and dist.is_initialized() else None


def world_size() -> int:
    dist = _distributed()
    return dist.get_world_size() if dist is not None else 1


def barrier() -> None:
    """Host barrier across ranks (no-op for a single process)."""
    dist = _distributed()
    if dist is not None and dist.get_world_size() > 1:
        dist.barrier()


def max_over_ranks(value: float, device=None) -> float:
    """Max of a per-rank measurement (timings are reported as the slowest
    rank's).  ``device`` is where the backend reduces (a CUDA device for
    NCCL; None for gloo on the host)."""
    dist = _distributed()
    if dist is None or dist.get_world_size() == 1:
        return float(value)
    import torch

    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(value: float, device=None) -> float:
    """Sum of a per-rank count (e.g. parity mismatches found by each rank)."""
    dist = _distributed()
    if dist is None or dist.get_world_size() == 1:
        return float(value)
    import torch

    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def gather_over_ranks(value) -> list:
    """Every rank's value, in rank order (a list of one for a single process)."""
    dist = _distributed()
    if dist is None or dist.get_world_size() == 1:
        return [value]
    out = [None] * dist.get_world_size()
    dist.all_gather_object(out, value)
    return out
