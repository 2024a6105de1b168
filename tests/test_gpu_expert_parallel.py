"""GPU, two or more devices: moe64a2 with experts split over the ranks (each rank holds
only its 64 / world experts; routed rows and results travel over NVLink peer memory) gives,
on each rank's positions, exactly the single-GPU forward's outputs."""

from __future__ import annotations

import multiprocessing as mp
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gpus() -> int:
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


@pytest.mark.parametrize(
    "world,d,depth,batch,repeats",
    [
        pytest.param(2, 256, 2, 700, 1),
        pytest.param(2, 768, 4, 4096, 3),
        # 8 experts a GPU, the expert split the c3 configuration names.
        pytest.param(8, 768, 4, 2048, 2, marks=pytest.mark.skipif(_gpus() < 8, reason="needs 8 GPUs")),
    ],
)
def test_expert_parallel_forward_equals_single_gpu(world: int, d: int, depth: int, batch: int, repeats: int) -> None:
    from ce4b200 import Moe64A2ChessNet, Moe64A2ChessNetConfig, _lib, replicas, synthetic
    from dist_worker import collect, ep_forward_worker

    if _gpus() < 2:
        pytest.skip("needs 2 GPUs")
    unique_id = _lib.nccl_unique_id()
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=ep_forward_worker, args=(r, world, port, unique_id, batch, queue, d, depth, repeats))
             for r in range(world)]
    try:
        for p in procs:
            p.start()
        results = sorted(collect(procs, queue, 600), key=lambda x: x[0])
        for p in procs:
            p.join(timeout=120)
            assert p.exitcode == 0
    finally:
        for p in procs:  # a rank left waiting on its peer is ended on the host
            if p.is_alive():
                p.kill()

    model = Moe64A2ChessNet(Moe64A2ChessNetConfig(d_model=d, depth=depth, expansion_ratio=1.0, precision="bf16"))
    weights = synthetic.make_moe_weights(d_model=d, depth=depth, expert_hidden=d, seed=5)
    synthetic.load_into(model, weights)
    model = model.cuda()
    planes = synthetic.lc0_to_dense(synthetic.make_lc0_planes(batch, 9))
    ref = model(planes.cuda())
    torch.cuda.synchronize()
    expert_bytes = sum(t.numel() * t.element_size() for k, t in weights.items() if ".experts." in k)
    for rank, policy, wdl, ml, tokens, full_bytes, held_bytes, code, same in results:
        assert code == 0, f"rank {rank}: device error word {code}"
        assert same, f"rank {rank}: repeated forwards differ"
        start, count = replicas.shard_rows(batch, world, rank)
        assert torch.equal(policy, ref.policy_logits.cpu()[start:start + count])
        assert torch.equal(wdl, ref.wdl_logits.cpu()[start:start + count])
        assert torch.equal(ml, ref.moves_left.cpu()[start:start + count])
        # Only this rank's experts stay resident.
        assert full_bytes - held_bytes >= expert_bytes * (world - 1) // world - 4096 * depth
    # Tokens per expert count this rank's own tokens; the ranks add up to the total.
    total = sum(r[4] for r in results)
    assert torch.equal(total, ref.router_tokens_per_expert.cpu())
