"""GPU: legal-move policy (softmax of the gathered logits times temperature, the lc0
backend's post-processing) on the device, against the CPU restatement."""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _moves(batch: int, seed: int, policy_size: int = 1858):
    g = np.random.default_rng(seed)
    counts = g.integers(0, 80, size=batch)
    counts[::17] = 0  # positions without legal moves
    counts[5] = 218   # the largest legal-move count in chess
    offsets = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
    indices = np.concatenate([g.choice(policy_size, size=c, replace=False) for c in counts]).astype(np.int32)
    return offsets, indices


@pytest.mark.parametrize("temperature", [1.0, 0.5, 2.2])
def test_policy_softmax_op_matches_restatement(temperature: float) -> None:
    from ce4b200 import kernels
    from oracle import policy as oracle

    batch = 300
    g = torch.Generator().manual_seed(3)
    logits = torch.randn(batch, 1858, generator=g) * 3
    offsets, indices = _moves(batch, 4)
    probs = kernels.policy_softmax(logits.cuda(), torch.from_numpy(offsets), torch.from_numpy(indices), temperature)
    torch.cuda.synchronize()
    ref = oracle.legal_move_softmax(logits.numpy(), offsets, indices, temperature)
    np.testing.assert_allclose(probs.cpu().numpy(), ref, rtol=2e-6, atol=1e-7)


def test_engine_evaluate_legal_matches_full_evaluate(tmp_path) -> None:
    from ce4b200 import DenseChessNet, DenseChessNetConfig, Engine, export_model, synthetic
    from oracle import policy as oracle

    model = DenseChessNet(DenseChessNetConfig(d_model=128, depth=2, expansion_ratio=3.0))
    synthetic.load_into(model, synthetic.make_dense_weights(d_model=128, depth=2, hidden_dim=384, seed=8))
    path = tmp_path / "m.safetensors"
    export_model(model, path)
    engine = Engine.load(path, gpu=0, max_batch=256)
    batch = 200
    planes = synthetic.lc0_planes_tensor(synthetic.make_lc0_planes(batch, 21))
    offsets, indices = _moves(batch, 22)
    probs, wdl, ml = engine.evaluate_legal(planes, torch.from_numpy(offsets), torch.from_numpy(indices), 1.3)
    policy, wdl_full, ml_full = engine.evaluate(planes)
    assert torch.equal(wdl, wdl_full) and torch.equal(ml, ml_full)
    ref = oracle.legal_move_softmax(policy.numpy(), offsets, indices, 1.3)
    np.testing.assert_allclose(probs.numpy(), ref, rtol=2e-6, atol=1e-7)
    for b in range(batch):
        lo, hi = offsets[b], offsets[b + 1]
        if hi > lo:
            assert abs(float(probs[lo:hi].sum()) - 1.0) < 1e-5
    with pytest.raises(ValueError):
        engine.evaluate_legal(planes, torch.from_numpy(offsets[:-1]), torch.from_numpy(indices))
