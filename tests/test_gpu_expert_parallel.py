"""GPU, two or more devices: moe64a2 with experts split over two ranks (NCCL send/recv of
routed rows) gives, on each rank's positions, exactly the single-GPU forward's outputs."""

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


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_expert_parallel_forward_equals_single_gpu() -> None:
    from ce4b200 import Moe64A2ChessNet, Moe64A2ChessNetConfig, _lib, replicas, synthetic
    from dist_worker import collect, ep_forward_worker

    batch = 700
    unique_id = _lib.nccl_unique_id()
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=ep_forward_worker, args=(r, 2, port, unique_id, batch, queue)) for r in range(2)]
    try:
        for p in procs:
            p.start()
        results = sorted(collect(procs, queue, 300), key=lambda x: x[0])
        for p in procs:
            p.join(timeout=120)
            assert p.exitcode == 0
    finally:
        for p in procs:  # a rank left waiting on its peer is ended on the host
            if p.is_alive():
                p.kill()

    model = Moe64A2ChessNet(Moe64A2ChessNetConfig(d_model=256, depth=2, expansion_ratio=1.0, precision="bf16"))
    synthetic.load_into(model, synthetic.make_moe_weights(d_model=256, depth=2, expert_hidden=256, seed=5))
    model = model.cuda()
    planes = synthetic.lc0_to_dense(synthetic.make_lc0_planes(batch, 9))
    ref = model(planes.cuda())
    torch.cuda.synchronize()
    for rank, policy, wdl, ml, tokens in results:
        start, count = replicas.shard_rows(batch, 2, rank)
        assert torch.equal(policy, ref.policy_logits.cpu()[start:start + count])
        assert torch.equal(wdl, ref.wdl_logits.cpu()[start:start + count])
        assert torch.equal(ml, ref.moves_left.cpu()[start:start + count])
    # Tokens per expert count this rank's own tokens; the two ranks add up to the total.
    if results[0][4] is not None and ref.router_tokens_per_expert is not None:
        total = results[0][4] + results[1][4]
        assert torch.equal(total, ref.router_tokens_per_expert.cpu())
