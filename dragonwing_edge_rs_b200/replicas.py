"""Batch-sharded replicas across GPUs (one process per GPU).

Whole-graph inference shards by image: every rank holds a full graph replica
and runs its contiguous slice of the global batch; nothing is exchanged on the
data path.  torch.distributed is used only on the host side: a barrier, the
max over ranks of a timing, and the exchange of per-rank status codes so that
a failed rank is reported by every rank instead of leaving the others waiting
(the reference propagates `Result` errors the same way,
crates/dragonwing-cpu/src/lib.rs:314-336).
"""
from __future__ import annotations

from dataclasses import dataclass

from . import _lib as L


def shard(global_batch: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous slice (start, count) of `global_batch` images for `rank`:
    floor(B/world) each, the remainder going to the last ranks."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world {world}")
    base, rem = divmod(global_batch, world)
    first_big = world - rem
    if rank < first_big:
        return rank * base, base
    return first_big * base + (rank - first_big) * (base + 1), base + 1


@dataclass
class RankStatus:
    rank: int
    status: int
    message: str = ""

    @property
    def ok(self) -> bool:
        return self.status == L.DW_OK


def exchange_status(dist, status: int, message: str = "") -> list[RankStatus]:
    """Every rank contributes its dw_status; every rank receives all of them.
    With no process group (single GPU), returns this rank's status alone."""
    if dist is None or not dist.is_initialized():
        return [RankStatus(0, status, message)]
    world = dist.get_world_size()
    gathered = [None] * world
    dist.all_gather_object(gathered, (int(status), str(message)))
    return [RankStatus(r, s, m) for r, (s, m) in enumerate(gathered)]


def max_over_ranks(dist, value: float, device=None) -> float:
    """Max of a host float over all ranks (device-timed regions are reported as
    the slowest rank's time)."""
    if dist is None or not dist.is_initialized():
        return value
    import torch
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(dist, value: int, device=None) -> int:
    if dist is None or not dist.is_initialized():
        return value
    import torch
    t = torch.tensor([int(value)], dtype=torch.int64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return int(t.item())
