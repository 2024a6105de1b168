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


def ep_plan_worker(rank: int, world: int, port: int, seed: int, queue) -> None:
    """Each rank routes random tokens, shares its per-expert segment sizes with all_gather
    (gloo), and plans its exchange with ce4b_expert_parallel_plan."""

    import ctypes

    import torch
    import torch.distributed as dist

    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from ce4b200 import _lib

    g = torch.Generator().manual_seed(seed + rank)
    counts = torch.randint(0, 300, (64,), generator=g, dtype=torch.int32)
    counts[torch.randint(0, 64, (8,), generator=g)] = 0
    meta = torch.stack([(counts + 127) // 128 * 128, counts], dim=1).to(torch.int32).contiguous()
    gathered = [torch.empty_like(meta) for _ in range(world)]
    dist.all_gather(gathered, meta)
    e_loc = 64 // world
    meta_recv = torch.cat([m[rank * e_loc:(rank + 1) * e_loc] for m in gathered]).contiguous()
    send = (ctypes.c_int32 * world)()
    recv = (ctypes.c_int32 * world)()
    tiles = (ctypes.c_int32 * (4 * 4096))()
    nt = ctypes.c_int()
    _lib.check(_lib.library().ce4b_expert_parallel_plan(
        world, rank, meta.data_ptr(), meta_recv.data_ptr(), send, recv, tiles, 4096, ctypes.byref(nt)))
    plan = (list(send), list(recv), [list(tiles[4 * i:4 * i + 4]) for i in range(nt.value)])
    both = [None] * world
    dist.all_gather_object(both, plan)
    queue.put((rank, both, meta_recv.tolist()))
    dist.destroy_process_group()


def ep_forward_worker(rank: int, world: int, port: int, unique_id: bytes, batch: int, queue,
                      d: int = 256, depth: int = 2, repeats: int = 1) -> None:
    """One expert-parallel rank on GPU `rank`: forwards its share of the batch `repeats`
    times (every result must be the same) and reports the weight bytes it holds before and
    after enabling expert parallelism."""

    import ctypes

    import torch

    torch.cuda.set_device(rank)
    from ce4b200 import Moe64A2ChessNet, Moe64A2ChessNetConfig, _lib, replicas, synthetic

    model = Moe64A2ChessNet(Moe64A2ChessNetConfig(d_model=d, depth=depth, expansion_ratio=1.0, precision="bf16"))
    synthetic.load_into(model, synthetic.make_moe_weights(d_model=d, depth=depth, expert_hidden=d, seed=5))
    model = model.cuda()
    planes = synthetic.lc0_to_dense(synthetic.make_lc0_planes(batch, 9))
    start, count = replicas.shard_rows(batch, world, rank)
    engine = model._engine(batch, torch.device("cuda", rank))
    info = _lib.ModelInfoStruct()
    _lib.check(engine.lib.ce4b_model_info_get(engine.handle, ctypes.byref(info)))
    full_bytes = info.weight_bytes
    model.enable_expert_parallel(max_batch=batch, rank=rank, world=world, unique_id=unique_id)
    _lib.check(engine.lib.ce4b_model_info_get(engine.handle, ctypes.byref(info)))
    outs = []
    for _ in range(repeats):
        out = model(planes[start:start + count].cuda())
        torch.cuda.synchronize()
        outs.append((out.policy_logits.cpu(), out.wdl_logits.cpu(), out.moves_left.cpu()))
    code = _lib.check_device_error(rank)
    same = all(torch.equal(a, b) for o in outs[1:] for a, b in zip(o, outs[0]))
    queue.put((rank, *outs[0],
               out.router_tokens_per_expert.cpu() if out.router_tokens_per_expert is not None else None,
               full_bytes, info.weight_bytes, code, same))


def collect(procs, queue, timeout_s: float):
    """One result per process; stops early (RuntimeError) when a process has exited
    without producing its result."""

    import queue as queue_mod
    import time

    results = []
    deadline = time.monotonic() + timeout_s
    while len(results) < len(procs):
        try:
            results.append(queue.get(timeout=1.0))
        except queue_mod.Empty:
            if any(p.exitcode not in (None, 0) for p in procs):
                raise RuntimeError(f"worker failed: exit codes {[p.exitcode for p in procs]}")
            if time.monotonic() > deadline:
                raise RuntimeError("workers timed out")
    return results
