"""Sharding independent segments over the GPUs of one node: one process per GPU.

wavo's long-audio path runs the pieces that src/split.rs cut at pauses one after another
(src/lib.rs:844-900); the pieces share nothing, so they partition across devices with no exchange
on the data path. Every rank builds the same `ShardPlan` (longest processing time first through
`wavo_partition_lpt`, deterministic), runs its own segments as varlen launches on its own stream,
and copies each segment's output rows to the host. `HostGather` puts every rank's segment rows
straight into one node-wide host buffer in the original segment order (the order wavo
concatenates transcripts in), each GPU over its own host link; `gather_in_order` does the same
through the process group's object gather where shared memory is short. The only cross-rank
traffic is a barrier and `max_over_ranks` of the step timings.
"""

from __future__ import annotations

import os
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


class HostGather:
    """The segment outputs of every rank of one node, in segment order, in one host buffer.

    Rank 0 creates a shared-memory buffer of Σ len rows of `width` values; every rank maps it,
    registers it with CUDA (page-locked, so device-to-host copies run asynchronously at full PCIe
    rate), and copies each of its own segments' rows from its packed device output straight to the
    segment's place — each GPU over its own host link, nothing between GPUs. After `wait` (the
    copies done on every rank, then a barrier) rank 0 reads every segment's output in segment
    order from `rows()`; `segment(i)` is segment i's rows. With one rank the buffer is private.

    When the node's shared memory cannot hold the buffer, `available` is False and the caller
    falls back to `gather_in_order`.
    """

    def __init__(self, plan: ShardPlan, lengths: Sequence[int], width: int, rank: int,
                 order: Sequence[int] | None = None, group=None):
        import numpy as np
        import torch

        self.plan, self.rank, self.group = plan, rank, group
        self.lengths = [int(t) for t in lengths]
        self.width = int(width)
        self.order = list(order) if order is not None else plan.mine(rank)
        if sorted(self.order) != plan.mine(rank):
            raise ValueError(f"rank {rank}: the order lists other segments than the plan gives it")
        self.offsets = [0]
        for t in self.lengths:
            self.offsets.append(self.offsets[-1] + t)
        total = self.offsets[-1]
        nbytes = max(total * self.width * 4, 4)
        self._shm = None
        self._registered = None
        self.available = True
        if plan.world > 1:
            import torch.distributed as dist
            from multiprocessing import shared_memory
            name = [None]
            if rank == 0:
                st = os.statvfs("/dev/shm") if os.path.isdir("/dev/shm") else None
                if st is None or st.f_bavail * st.f_frsize < nbytes + (64 << 20):
                    name[0] = ""
                else:
                    self._shm = shared_memory.SharedMemory(create=True, size=nbytes)
                    name[0] = self._shm.name
            dist.broadcast_object_list(name, src=0, group=group)
            if not name[0]:
                self.available = False
                return
            if rank != 0:
                self._shm = shared_memory.SharedMemory(name=name[0])
                # Rank 0 created the segment and removes it; the others only map it.
                from multiprocessing import resource_tracker
                resource_tracker.unregister(self._shm._name, "shared_memory")
            buf = np.ndarray((total, self.width), np.float32, buffer=self._shm.buf)
            self.host = torch.from_numpy(buf)
        else:
            self.host = torch.empty((total, self.width), dtype=torch.float32)
        if torch.cuda.is_available():
            if plan.world > 1:
                err = torch.cuda.cudart().cudaHostRegister(self.host.data_ptr(), nbytes, 0)
                if int(err) != 0:
                    raise RuntimeError(f"cudaHostRegister of the shared output: error {int(err)}")
                self._registered = self.host.data_ptr()
            else:
                self.host = self.host.pin_memory()
        # (packed row, output row, rows) of each of this rank's segments; adjacent runs merged.
        runs, at = [], 0
        for i in self.order:
            t = self.lengths[i]
            if runs and runs[-1][0] + runs[-1][2] == at and runs[-1][1] + runs[-1][2] == \
                    self.offsets[i]:
                runs[-1][2] += t
            else:
                runs.append([at, self.offsets[i], t])
            at += t
        self.runs = [tuple(r) for r in runs]
        self.packed_rows = at

    def copy_from(self, packed) -> None:
        """Enqueues the copies of this rank's packed output rows ([Σ its len][width], in `order`)
        to their places (device tensors: asynchronous on the current stream)."""
        if packed.shape[0] != self.packed_rows or packed.shape[1] != self.width:
            raise ValueError(f"packed output {tuple(packed.shape)}, expected "
                             f"({self.packed_rows}, {self.width})")
        nb = packed.is_cuda
        for src, dst, n in self.runs:
            self.host[dst:dst + n].copy_(packed[src:src + n], non_blocking=nb)

    def wait(self, stream=None) -> None:
        """The copies of every rank have landed: this rank's stream drained, then a barrier."""
        import torch
        if torch.cuda.is_available():
            (stream or torch.cuda.current_stream()).synchronize()
        if self.plan.world > 1:
            import torch.distributed as dist
            dist.barrier(group=self.group)

    def rows(self):
        """All segments' rows in segment order (rank 0, after `wait`)."""
        return self.host

    def segment(self, i: int):
        return self.host[self.offsets[i]:self.offsets[i + 1]]

    def close(self) -> None:
        import torch
        if self._registered is not None:
            torch.cuda.cudart().cudaHostUnregister(self._registered)
            self._registered = None
        self.host = None
        if self._shm is not None:
            self._shm.close()
            if self.rank == 0:
                self._shm.unlink()
            self._shm = None
