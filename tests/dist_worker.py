"""Worker for the gloo multi-process tests (spawned; importable by module name)."""

from __future__ import annotations

import os


def replica_worker(rank: int, world: int, port: int, total: int, queue) -> None:
    os.environ.update(RANK=str(rank), LOCAL_RANK=str(rank), WORLD_SIZE=str(world),
                      MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from ce4b200 import replicas

    group = replicas.init_from_env(backend="gloo", timeout_s=60)
    start, count = replicas.shard_rows(total, world, rank)
    slowest = group.max(float(10 * rank + 1))
    covered = group.sum(float(count))
    group.barrier()
    queue.put((rank, start, count, slowest, covered, str(group.device)))
    group.close()
