"""Data-parallel plumbing for the batch-sharded path (one process per GPU).

The path has no data exchange: utterances are independent, weights are
replicated, and each rank quantizes, multiplies and filters its own shard.  The
only collectives are the start barrier and the max-reduction of the measured
time, both off the data path.
"""
from __future__ import annotations

import os
from dataclasses import dataclass
from datetime import timedelta


def shard_range(total: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous [start, stop) share of `total` units for `rank` (sizes differ by at most one)."""
    if world <= 0 or not 0 <= rank < world or total < 0:
        raise ValueError("invalid shard request")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


@dataclass
class RankContext:
    rank: int
    world: int
    local_rank: int
    backend: str
    initialized: bool = False

    @classmethod
    def from_env(cls, backend: str = "nccl") -> "RankContext":
        return cls(int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
                   int(os.environ.get("LOCAL_RANK", "0")), backend)

    def init(self, timeout_s: float = 300.0, device=None) -> "RankContext":
        """Join the process group (only when world > 1)."""
        if self.world > 1 and not self.initialized:
            import torch.distributed as dist
            kwargs = {"timeout": timedelta(seconds=timeout_s)}
            if device is not None and self.backend == "nccl":
                kwargs["device_id"] = device
            dist.init_process_group(self.backend, **kwargs)
            self.initialized = True
        return self

    def barrier(self) -> None:
        if self.initialized:
            import torch.distributed as dist
            dist.barrier()

    def max_over_ranks(self, value: float, device=None) -> float:
        """The slowest rank's value (the job finishes when the last rank does)."""
        if not self.initialized:
            return float(value)
        import torch
        import torch.distributed as dist
        t = torch.tensor([float(value)], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def close(self) -> None:
        if self.initialized:
            import torch.distributed as dist
            dist.destroy_process_group()
            self.initialized = False


def weak_scaling_throughput(work_per_rank: float, world: int, slowest_seconds: float) -> float:
    """Whole-job rate: every rank processes `work_per_rank`; the job ends with the slowest rank."""
    if slowest_seconds <= 0:
        raise ValueError("elapsed time must be positive")
    return world * work_per_rank / slowest_seconds


def strong_scaling_throughput(total_work: float, slowest_seconds: float) -> float:
    """Whole-job rate of a fixed batch split over the ranks: the job ends with the slowest rank."""
    if slowest_seconds <= 0:
        raise ValueError("elapsed time must be positive")
    return total_work / slowest_seconds
