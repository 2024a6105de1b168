"""Data-parallel replicas of the forward, one process per GPU.

Positions are independent, so a multi-GPU forward of a dense (or replicated moe64a2)
model is N independent replicas, each evaluating a contiguous slice of the batch on its
own GPU with its own copy of the weights; no collective touches the data path. The
process group (NCCL on GPUs, gloo on CPU) only starts the ranks together and reduces
timings. Launch with ``torchrun --nproc-per-node N`` (``RANK``, ``LOCAL_RANK``,
``WORLD_SIZE``, ``MASTER_ADDR`` / ``MASTER_PORT`` from the environment).
"""

from __future__ import annotations

import datetime
import os
from dataclasses import dataclass

import torch


def shard_rows(total: int, world: int, rank: int) -> tuple[int, int]:
    """(start, count) of rank's contiguous slice of ``total`` positions; the first
    ``total % world`` ranks take one more position."""

    if world < 1 or not 0 <= rank < world or total < 0:
        raise ValueError(f"bad shard request total={total} world={world} rank={rank}")
    base, extra = divmod(total, world)
    count = base + (1 if rank < extra else 0)
    start = rank * base + min(rank, extra)
    return start, count


@dataclass
class ReplicaGroup:
    world: int
    rank: int
    local_rank: int
    backend: str | None  # None when world == 1 (no process group)

    @property
    def device(self) -> torch.device:
        if self.backend == "nccl" or (self.backend is None and torch.cuda.is_available()):
            return torch.device("cuda", self.local_rank)
        return torch.device("cpu")

    def barrier(self) -> None:
        if self.backend is not None:
            import torch.distributed as dist

            dist.barrier()

    def _reduce(self, value: float, op_name: str) -> float:
        if self.backend is None:
            return value
        import torch.distributed as dist

        op = getattr(dist.ReduceOp, op_name)
        t = torch.tensor([value], dtype=torch.float64, device=self.device)
        dist.all_reduce(t, op=op)
        return float(t.item())

    def max(self, value: float) -> float:
        """Maximum over ranks (every rank must call it; the slowest rank's time)."""

        return self._reduce(value, "MAX")

    def sum(self, value: float) -> float:
        return self._reduce(value, "SUM")

    def close(self) -> None:
        if self.backend is not None:
            import torch.distributed as dist

            dist.destroy_process_group()
            self.backend = None


def init_from_env(backend: str | None = None, timeout_s: float = 120.0) -> ReplicaGroup:
    """Joins the torchrun process group (NCCL if CUDA is available, else gloo). With
    WORLD_SIZE unset or 1 no process group is created."""

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world <= 1:
        return ReplicaGroup(1, 0, local, None)
    import torch.distributed as dist

    if backend is None:
        backend = "nccl" if torch.cuda.is_available() else "gloo"
    timeout = datetime.timedelta(seconds=timeout_s)
    if backend == "nccl":
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timeout, device_id=torch.device("cuda", local))
    else:
        dist.init_process_group(backend, timeout=timeout)
    return ReplicaGroup(world, rank, local, backend)
