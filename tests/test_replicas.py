"""Multi-GPU host logic on CPU: batch shards and the replica process group (gloo,
world size 2), as bench.py uses them under torchrun."""

from __future__ import annotations

import multiprocessing as mp
import socket

import pytest


@pytest.mark.parametrize("total,world", [(4096, 1), (4096, 2), (16384, 8), (65536, 8), (7, 3), (0, 2)])
def test_shards_are_contiguous_and_cover_the_batch(total: int, world: int) -> None:
    from ce4b200 import replicas

    shards = [replicas.shard_rows(total, world, r) for r in range(world)]
    assert sum(c for _, c in shards) == total
    pos = 0
    for start, count in shards:
        assert start == pos and count >= 0
        pos += count
    counts = [c for _, c in shards]
    assert max(counts) - min(counts) <= 1
    with pytest.raises(ValueError):
        replicas.shard_rows(total, world, world)


def test_single_process_group_needs_no_backend(monkeypatch) -> None:
    from ce4b200 import replicas

    monkeypatch.delenv("WORLD_SIZE", raising=False)
    group = replicas.init_from_env()
    assert group.world == 1 and group.backend is None
    assert group.max(3.5) == 3.5 and group.sum(2.0) == 2.0
    group.barrier()
    group.close()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_rank_replica_group_on_gloo() -> None:
    from dist_worker import collect, replica_worker

    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=replica_worker, args=(r, 2, port, 4097, queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = sorted(collect(procs, queue, 120))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    (r0, s0, c0, m0, t0, d0), (r1, s1, c1, m1, t1, d1) = results
    assert (s0, c0, s1, c1) == (0, 2049, 2049, 2048)
    assert m0 == m1 == 11.0  # max over ranks of 10 * rank + 1
    assert t0 == t1 == 4097.0
    assert d0 == d1 == "cpu"
