"""Sharding independent segments over the GPUs of one node: one process per GPU.

wavo's long-audio path runs the pieces that src/split.rs cut at pauses one after another
(src/lib.rs:844-900); the pieces share nothing, so they partition across devices with no exchange
on the data path. Every rank builds the same `ShardPlan` (longest processing time first through
`wavo_partition_lpt`, deterministic), runs its own segments as varlen launches on its own stream,
and copies each segment's output rows to the host. `gather_in_order` then hands rank 0 every
segment's output in the original segment order, the order wavo concatenates transcripts in.
The only cross-rank traffic is that host-side gather and `max_over_ranks` of the step timings.
"""

from __future__ import annotations

from typing import Callable, Sequence

from .gpu import partition_lpt


def encoder_cost(t: int, d: int, layers: int) -> int:
    """Relative cost of one segment of `t` frames through `layers` attention layers of width `d`:
    the attention core (6·T²·d for the relative-position form) plus the projections (10·T·d²)."""
    return layers * (6 * t * t * d + 10 * t * d * d)


class ShardPlan:
    """Which rank runs which segment. The same inputs give the same plan on every rank."""

    def __init__(self, costs: Sequence[int], world: int):
        if world < 1:
            raise ValueError("world must be at least 1")
        self.world = world
        self.costs = [int(c) for c in costs]
        self.assign = partition_lpt(self.costs, world) if world > 1 and self.costs else \
            [0] * len(self.costs)

    @classmethod
    def for_lengths(cls, lengths: Sequence[int], world: int,
                    cost: Callable[[int], int]) -> "ShardPlan":
        return cls([cost(t) for t in lengths], world)

    def mine(self, rank: int) -> list[int]:
        """The segments `rank` runs, in their original order."""
        if not 0 <= rank < self.world:
            raise ValueError(f"rank {rank} outside a world of {self.world}")
        return [i for i, a in enumerate(self.assign) if a == rank]

    def launch_order(self, rank: int) -> list[int]:
        """The segments `rank` runs, costliest first: the order to pack them in. The attention
        kernels take a launch's segments in packed order (the flash kernel's CTAs are dispatched
        in that order, the persistent kernel deals its items round-robin in it), so the long
        segments start first and the short ones fill the tail (C3: 1.910 -> 1.888 ms a step,
        C5: 29.88 -> 29.45 ms on one B200)."""
        return sorted(self.mine(rank), key=lambda i: (-self.costs[i], i))

    def loads(self) -> list[int]:
        """Total cost per rank."""
        out = [0] * self.world
        for c, a in zip(self.costs, self.assign):
            out[a] += c
        return out


def split_rows(rows, lengths: Sequence[int]) -> list:
    """Cut a packed `[Σ len][d]` output (segments one after another) into per-segment pieces."""
    out, at = [], 0
    for t in lengths:
        out.append(rows[at:at + t])
        at += t
    if at != len(rows):
        raise ValueError(f"{len(rows)} rows for segments of {at} frames in total")
    return out


def gather_in_order(plan: ShardPlan, rank: int, outputs: Sequence, group=None,
                    order: Sequence[int] | None = None):
    """Rank 0 receives every segment's output in segment order; other ranks get None.

    `outputs` holds this rank's host arrays, one per segment of `order` (by default
    `plan.mine(rank)`; `plan.launch_order(rank)` when the segments were packed in that order), in
    that order. With one rank nothing crosses processes. The gather goes through the process
    group's object gather, on the host: it is off the device data path and outside any timed
    region.
    """
    mine = list(order) if order is not None else plan.mine(rank)
    if sorted(mine) != plan.mine(rank):
        raise ValueError(f"rank {rank}: the order lists other segments than the plan gives it")
    if len(outputs) != len(mine):
        raise ValueError(f"rank {rank} runs {len(mine)} segments but passed {len(outputs)} outputs")
    if plan.world == 1:
        ordered = [None] * len(plan.assign)
        for i, o in zip(mine, outputs):
            ordered[i] = o
        return ordered
    import torch.distributed as dist
    parts = [None] * plan.world if rank == 0 else None
    dist.gather_object((list(mine), list(outputs)), parts, dst=0, group=group)
    if rank != 0:
        return None
    ordered = [None] * len(plan.assign)
    for segs, outs in parts:
        for i, o in zip(segs, outs):
            ordered[i] = o
    missing = [i for i, o in enumerate(ordered) if o is None]
    if missing:
        raise RuntimeError(f"segments {missing[:8]} came back from no rank")
    return ordered


def max_over_ranks(values: Sequence[float], device=None, group=None) -> list[float]:
    """Element-wise maximum over the ranks (the step time of the slowest rank)."""
    import torch
    import torch.distributed as dist
    t = torch.tensor(list(values), dtype=torch.float64, device=device)
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return t.tolist()
