"""Request-batch data parallelism: each rank owns a disjoint slice of the
sequences and its own KV pages; the only cross-rank traffic is the acceptance
counters (SpecDiagnosticCounters, include/engine/speculative_verifier.hpp:31-53)
summed with one all_reduce.
"""
from __future__ import annotations

import datetime
import os
from typing import Dict, Optional, Tuple

import torch
import torch.distributed as dist

from ._lib import STAT_NAMES


def shard(global_batch: int, rank: int, world: int) -> Tuple[int, int]:
    """Contiguous [start, stop) of the sequences owned by `rank`."""
    base, rem = divmod(global_batch, world)
    start = rank * base + min(rank, rem)
    return start, start + base + (1 if rank < rem else 0)


def init(backend: str = "nccl", timeout_s: float = 120.0):
    """Process group from torchrun's environment (no-op for a single process)."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1 and not dist.is_initialized():
        kw = dict(timeout=datetime.timedelta(seconds=timeout_s))
        if backend == "nccl":
            kw["device_id"] = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
        dist.init_process_group(backend, **kw)
    return (dist.get_rank(), dist.get_world_size()) if dist.is_initialized() else (0, 1)


def reduce_stats(stats: torch.Tensor) -> torch.Tensor:
    """Sum of every rank's int64 counters (a copy; `stats` is untouched)."""
    out = stats.clone()
    if dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(out, op=dist.ReduceOp.SUM)
    return out


def max_time(ms: float, device=None) -> float:
    """Max over ranks of a per-rank device time (the job's wall time on the GPUs)."""
    if not (dist.is_initialized() and dist.get_world_size() > 1):
        return ms
    t = torch.tensor([ms], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def stats_dict(stats: torch.Tensor) -> Dict[str, int]:
    return dict(zip(STAT_NAMES, stats.cpu().tolist()))


class CounterReducer:
    """The acceptance counters summed over the ranks every `every` steps, off
    the compute stream.

    `stats` is the int64 counter tensor the acceptance kernel accumulates on
    the device. Call step() once per decode step, after the step's kernels are
    enqueued: every `every` steps it snapshots the counters on the current
    stream and, on a side stream that waits only for that snapshot,
    all-reduces the snapshot, so the collective overlaps the following steps'
    kernels. Two snapshot buffers alternate, and one is rewritten only after the
    all-reduce that last read it. Every rank must call step() the same number
    of times (the collectives pair up in order). On CPU tensors (gloo) the
    all-reduce runs in line. finish() makes the current stream wait for the
    side stream; result() is the last reduced snapshot with the step it covers.
    """

    def __init__(self, stats: torch.Tensor, every: int = 5):
        self.stats = stats
        self.every = max(1, int(every))
        self.world = dist.get_world_size() if dist.is_initialized() else 1
        self.cuda = stats.is_cuda
        self.side = torch.cuda.Stream(device=stats.device) if (self.cuda and self.world > 1) else None
        self.snaps = [torch.zeros_like(stats) for _ in range(2)]
        self.read = [torch.cuda.Event(), torch.cuda.Event()] if self.side is not None else None
        self.taken = torch.cuda.Event() if self.side is not None else None
        self.steps = 0
        self.reduces = 0
        self.last: Optional[Tuple[int, int]] = None

    def step(self) -> None:
        k = self.steps
        self.steps += 1
        if self.world == 1 or k % self.every != self.every - 1:
            return
        j = self.reduces % 2
        if self.side is not None:
            cur = torch.cuda.current_stream(self.stats.device)
            if self.reduces >= 2:
                cur.wait_event(self.read[j])
            self.snaps[j].copy_(self.stats)
            self.taken.record(cur)
            self.side.wait_event(self.taken)
            with torch.cuda.stream(self.side):
                dist.all_reduce(self.snaps[j], op=dist.ReduceOp.SUM)
                self.read[j].record(self.side)
        else:
            self.snaps[j].copy_(self.stats)
            dist.all_reduce(self.snaps[j], op=dist.ReduceOp.SUM)
        self.reduces += 1
        self.last = (j, self.steps)

    def finish(self) -> None:
        if self.side is not None:
            torch.cuda.current_stream(self.stats.device).wait_stream(self.side)

    def result(self) -> Optional[Dict[str, int]]:
        if self.last is None:
            return None
        j, through = self.last
        out = stats_dict(self.snaps[j])
        out["through_step"] = through
        out["ranks"] = self.world
        return out
