"""GPU parity of the small-batch dense forward (batches of at most 64 positions, d_model <=
512): one cooperative launch of transposed tcgen05 tiles spread over the SMs, with the
persistent forward's folded RMSNorm (W' = bf16(W * diag(w)), the row's rsqrt(mean(x^2) +
eps) on the FP32 accumulator). Checked against the CPU restatement of the reference's BF16
forward (oracle/dense.py, mode="bf16": the full contract), against the restatement of the
folded arithmetic, against the persistent forward of the same model, and for determinism."""

from __future__ import annotations

import pytest
import torch

from helpers import (
    ARGMAX_AGREEMENT,
    POLICY_ATOL,
    POLICY_RTOL,
    WDL_PROB_ATOL,
    argmax_agreement,
    assert_policy_close,
    dense_model,
)

pytestmark = pytest.mark.gpu


def _case(d: int, depth: int, ratio: float, batch: int, hist: int = 8, seed: int = 0):
    from ce4b200 import synthetic

    weights = synthetic.make_dense_weights(
        d_model=d, depth=depth, hidden_dim=int(d * ratio), seed=seed, history_length=hist
    )
    planes = synthetic.lc0_to_dense(synthetic.make_lc0_planes(batch, seed + 11))
    return weights, planes


@pytest.mark.parametrize(
    "d,depth,ratio,batch,hist",
    [
        (512, 12, 3.0, 64, 8),  # the latency benchmark shape
        (512, 2, 3.0, 1, 8),  # one position (N = 16)
        (128, 6, 3.0, 17, 8),  # d128: one 128-row block, 112 input K parts
        (256, 4, 3.0, 48, 8),
        (512, 3, 2.0, 33, 8),  # h = 1024
        (384, 1, 3.0, 40, 2),  # one layer, short history (21 planes: 7 input K parts)
    ],
)
def test_small_batch_forward_matches_oracle(d: int, depth: int, ratio: float, batch: int, hist: int) -> None:
    from ce4b200 import _lib
    from oracle import dense as oracle

    weights, planes = _case(d, depth, ratio, batch, hist)
    model = dense_model(weights, d=d, depth=depth, ratio=ratio, hist=hist).cuda()
    out = model(planes.cuda())
    torch.cuda.synchronize()
    assert model._native.uses_latency_path(batch)
    assert _lib.check_device_error(0) == 0
    ref16 = oracle.forward(weights, planes, depth=depth, history_length=hist, mode="bf16")
    folded = oracle.forward(weights, planes, depth=depth, history_length=hist, mode="bf16", fold_norm=True)
    ours = out.policy_logits.cpu()
    assert_policy_close(ours, ref16[0], atol=POLICY_ATOL, rtol=POLICY_RTOL)
    raw = argmax_agreement(ours, ref16[0], tol=0.0)
    tol_aware = argmax_agreement(ours, ref16[0])
    mean_ref = float((ours - ref16[0]).abs().mean())
    mean_folded = float((ours - folded[0]).abs().mean())
    print(f"d{d}x{depth} B={batch}: max {float((ours - ref16[0]).abs().max()):.4g}, mean {mean_ref:.3g} "
          f"(folded restatement {mean_folded:.3g}), argmax raw {raw:.4f}, tolerance-aware {tol_aware:.4f}")
    # The kernel computes the folded arithmetic: it sits closer to that restatement than to
    # the reference's rounding points, and within the logit bar of it.
    assert mean_folded <= mean_ref
    assert float((ours - folded[0]).abs().max()) <= POLICY_ATOL
    assert tol_aware >= ARGMAX_AGREEMENT
    torch.testing.assert_close(
        torch.softmax(out.wdl_logits.cpu(), -1), oracle.wdl_probabilities(ref16[1]), atol=WDL_PROB_ATOL, rtol=0
    )
    torch.testing.assert_close(out.moves_left.cpu(), ref16[2], atol=POLICY_ATOL, rtol=POLICY_RTOL)


def test_small_batch_forward_is_deterministic_and_agrees_with_persistent() -> None:
    weights, planes = _case(512, 4, 3.0, 64, seed=3)
    model = dense_model(weights, d=512, depth=4, ratio=3.0).cuda()
    x = planes.cuda()
    first = model(x.clone())
    torch.cuda.synchronize()
    ref = [t.clone() for t in (first.policy_logits, first.wdl_logits, first.moves_left)]
    for _ in range(3):
        again = model(x.clone())
        torch.cuda.synchronize()
        for a, b in zip(ref, (again.policy_logits, again.wdl_logits, again.moves_left)):
            assert torch.equal(a, b)
    # Sub-batches: rows are independent and the K-split sums are in fixed order whatever N.
    for rows in (1, 16, 40):
        part = model(x[:rows].clone())
        torch.cuda.synchronize()
        for a, b in zip(ref, (part.policy_logits, part.wdl_logits, part.moves_left)):
            assert torch.equal(a[:rows], b)
    model.set_latency_path(False)
    assert not model._native.uses_latency_path(64)
    persistent = model(x.clone())
    torch.cuda.synchronize()
    # Same arithmetic, different FP32 accumulation order.
    torch.testing.assert_close(persistent.policy_logits, ref[0], atol=POLICY_ATOL, rtol=POLICY_RTOL)
    print("small-batch vs persistent: max", float((persistent.policy_logits - ref[0]).abs().max()))
    torch.testing.assert_close(
        torch.softmax(persistent.wdl_logits, -1), torch.softmax(ref[1], -1), atol=WDL_PROB_ATOL, rtol=0
    )


def test_small_batch_evaluate_through_the_c_abi(tmp_path) -> None:
    """lc0 InputPlane records through ce4b_model_evaluate (graph-captured forward, host
    buffers) at small batches equal the device forward of the same records, through the
    copy path (pageable buffers, or direct I/O off) and through the copy-free path (pinned
    buffers: the kernels read the records and write the outputs in host memory)."""

    from ce4b200 import DenseChessNet, DenseChessNetConfig, Engine, _lib, export_model, synthetic

    d, depth = 512, 3
    weights = synthetic.make_dense_weights(d_model=d, depth=depth, hidden_dim=3 * d, seed=6)
    model = DenseChessNet(DenseChessNetConfig(d_model=d, depth=depth, expansion_ratio=3.0, precision="bf16"))
    synthetic.load_into(model, weights)
    path = tmp_path / "m.safetensors"
    export_model(model, path)
    engine = Engine.load(path, gpu=0, max_batch=256)
    dm = model.cuda()
    for batch in (64, 23):
        lc0 = synthetic.lc0_planes_tensor(synthetic.make_lc0_planes(batch, 7 + batch))
        dev = dm.forward_lc0(lc0.cuda())
        torch.cuda.synchronize()
        expect = (dev.policy_logits.cpu(), dev.wdl_logits.cpu(), dev.moves_left.cpu())
        pinned_in = lc0.pin_memory()
        runs = []
        for direct in (True, False):
            engine.set_direct_io(direct)
            runs.append(engine.evaluate(lc0))  # pageable: copies
            for _ in range(2):
                out = engine.outputs(batch, pin=True)
                runs.append(engine.evaluate(pinned_in, out))  # pinned: copy-free when direct
            out = engine.outputs(batch, pin=True)
            for _ in range(3):  # the same buffers again (cached graph), then reset outputs
                for t in out:
                    t.fill_(float("nan"))
                runs.append(engine.evaluate(pinned_in, out))
        for got in runs:
            for x, y in zip(got, expect):
                assert torch.equal(x, y)
    assert _lib.check_device_error(0) == 0


@pytest.mark.parametrize("hist", [8, 2])
def test_small_batch_lc0_records_expanded_in_kernel_match_plane_layouts(hist: int) -> None:
    """lc0 InputPlane records and dense planes of the same positions give the same bits at
    a small batch (history selection and the rule-50 / 99 included)."""

    from ce4b200 import synthetic

    d, depth, batch = 256, 2, 40
    weights = synthetic.make_dense_weights(d_model=d, depth=depth, hidden_dim=3 * d, seed=8, history_length=hist)
    lc0 = synthetic.make_lc0_planes(batch, 13, aux_constant=True)
    model = dense_model(weights, d=d, depth=depth, ratio=3.0, hist=hist).cuda()
    a = model(synthetic.lc0_to_dense(lc0).cuda())
    e = model.forward_lc0(synthetic.lc0_planes_tensor(lc0).cuda(), wdl_probs=False)
    torch.cuda.synchronize()
    assert model._native.uses_latency_path(batch)
    for x, y in ((a.policy_logits, e.policy_logits), (a.wdl_logits, e.wdl_logits), (a.moves_left, e.moves_left)):
        assert torch.equal(x, y)


def test_small_batch_async_copy_free_and_copy_calls_interleave(tmp_path) -> None:
    """Small-batch evaluate_async calls on two streams, alternating the copy-free path
    (pinned buffers, kernels reading and writing host memory) and the copy path, give the
    blocking evaluate's results: the forwards share the model's workspace and are ordered
    across streams whichever path a call takes."""

    from ce4b200 import DenseChessNet, DenseChessNetConfig, Engine, _lib, export_model, synthetic

    d, depth = 256, 2
    weights = synthetic.make_dense_weights(d_model=d, depth=depth, hidden_dim=3 * d, seed=21)
    model = DenseChessNet(DenseChessNetConfig(d_model=d, depth=depth, expansion_ratio=3.0, precision="bf16"))
    synthetic.load_into(model, weights)
    path = tmp_path / "m.safetensors"
    export_model(model, path)
    engine = Engine.load(path, gpu=0, max_batch=256)
    sizes = [64, 48, 64, 17, 64, 30, 1, 64]
    batches = [synthetic.lc0_planes_tensor(synthetic.make_lc0_planes(b, 60 + i)).pin_memory()
               for i, b in enumerate(sizes)]
    expected = [engine.evaluate(p) for p in batches]  # pageable outputs: copy path
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    outs = [engine.outputs(int(p.shape[0]), pin=True) for p in batches]
    for rep in range(2):
        for o in outs:
            for t in o:
                t.fill_(float("nan"))
        for i, (p, o) in enumerate(zip(batches, outs)):
            engine.set_direct_io(i % 2 == rep)
            engine.evaluate_async(p, o, streams[i % 2])
        for s in streams:
            s.synchronize()
        for got, exp in zip(outs, expected):
            for x, y in zip(got, exp):
                assert torch.equal(x, y)
    engine.set_direct_io(True)
    assert _lib.check_device_error(0) == 0
    engine.close()
