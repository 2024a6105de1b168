"""Expert-parallel exchange planning on the host (no GPU): the C ABI's plan against a
restatement, and a gloo world-size-2 exchange of segment metadata whose send and receive
sizes must agree between the ranks."""

from __future__ import annotations

import ctypes
import multiprocessing as mp
import socket

import pytest
import torch


def _plan(world: int, rank: int, meta_send: torch.Tensor, meta_recv: torch.Tensor):
    from ce4b200 import _lib

    send = (ctypes.c_int32 * world)()
    recv = (ctypes.c_int32 * world)()
    tiles = (ctypes.c_int32 * (4 * 8192))()
    nt = ctypes.c_int()
    _lib.check(_lib.library().ce4b_expert_parallel_plan(
        world, rank, meta_send.data_ptr(), meta_recv.data_ptr(), send, recv, tiles, 8192, ctypes.byref(nt)))
    return list(send), list(recv), [tuple(tiles[4 * i:4 * i + 4]) for i in range(nt.value)]


def _restated(world: int, rank: int, meta_send: torch.Tensor, meta_recv: torch.Tensor):
    e_loc = 64 // world
    send = [int(meta_send[r * e_loc:(r + 1) * e_loc, 0].sum()) for r in range(world)]
    recv, tiles, row = [], [], 0
    for r in range(world):
        recv.append(int(meta_recv[r * e_loc:(r + 1) * e_loc, 0].sum()))
        for e in range(e_loc):
            padded, valid = (int(v) for v in meta_recv[r * e_loc + e])
            for i in range(0, valid, 128):
                tiles.append((rank * e_loc + e, row + i, min(128, valid - i), 0))
            row += padded
    return send, recv, tiles


def _meta(counts: torch.Tensor) -> torch.Tensor:
    return torch.stack([(counts + 127) // 128 * 128, counts], dim=1).to(torch.int32).contiguous()


@pytest.mark.parametrize("world,rank", [(2, 0), (2, 1), (4, 3), (8, 5)])
def test_plan_matches_restatement(world: int, rank: int) -> None:
    g = torch.Generator().manual_seed(world * 10 + rank)
    meta_send = _meta(torch.randint(0, 400, (64,), generator=g))
    e_loc = 64 // world
    meta_recv = _meta(torch.randint(0, 400, (world * e_loc,), generator=g))
    meta_recv[3] = 0  # an expert no token of that source chose
    assert _plan(world, rank, meta_send, meta_recv) == _restated(world, rank, meta_send, meta_recv)


def test_plan_rejects_bad_metadata() -> None:
    from ce4b200 import _lib

    meta = _meta(torch.full((64,), 5))
    bad = meta.clone()
    bad[0, 0] = 100  # not a multiple of 128
    with pytest.raises(ValueError):
        _plan(2, 0, meta, bad)
    with pytest.raises(ValueError):
        _plan(3, 0, meta, meta)  # 3 does not divide 64
    assert _lib.CE4B_ERR_INVALID_ARGUMENT != 0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_rank_exchange_sizes_agree_on_gloo() -> None:
    from dist_worker import collect, ep_plan_worker

    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=ep_plan_worker, args=(r, 2, port, 7, queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = sorted(collect(procs, queue, 120), key=lambda x: x[0])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    plans = results[0][1]
    assert plans == results[1][1]
    for a in range(2):
        for b in range(2):
            # rows rank a sends to rank b == rows rank b receives from rank a
            assert plans[a][0][b] == plans[b][1][a]
    for rank in range(2):
        tiles = plans[rank][2]
        assert all(rank * 32 <= t[0] < (rank + 1) * 32 and 0 < t[2] <= 128 and t[1] % 128 == 0 for t in tiles)
