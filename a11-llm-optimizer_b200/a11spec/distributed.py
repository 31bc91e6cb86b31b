"""Request-batch data parallelism: each rank owns a disjoint slice of the
sequences and its own KV pages; the only cross-rank traffic is the acceptance
counters (SpecDiagnosticCounters, include/engine/speculative_verifier.hpp:31-53)
summed with one all_reduce.
"""
from __future__ import annotations

import datetime
import os
from typing import Dict, Tuple

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
