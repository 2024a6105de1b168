"""GPU: the engine path (Safetensors v1 file -> ce4b_model_load_safetensors ->
ce4b_model_evaluate) against the oracle, and the pipelined evaluate_async against the
blocking call (mirrors Model::Load / Model::Evaluate,
kernels/include/chess_engine_4/inference.h:29-51)."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _dense(d: int, depth: int, seed: int):
    from ce4b200 import DenseChessNet, DenseChessNetConfig, synthetic

    weights = synthetic.make_dense_weights(d_model=d, depth=depth, hidden_dim=3 * d, seed=seed)
    model = DenseChessNet(DenseChessNetConfig(d_model=d, depth=depth, expansion_ratio=3.0))
    synthetic.load_into(model, weights)
    return model, weights


def test_engine_loads_exported_file_and_matches_oracle(tmp_path) -> None:
    from ce4b200 import Engine, export_model, synthetic
    from helpers import POLICY_ATOL, WDL_PROB_ATOL, argmax_agreement
    from oracle import dense as oracle

    model, weights = _dense(128, 3, seed=11)
    path = tmp_path / "dense.safetensors"
    export_model(model, path)
    engine = Engine.load(path, gpu=0, max_batch=512)
    assert engine.info.d_model == 128 and engine.info.depth == 3 and engine.info.maximum_batch_size == 512
    lc0 = synthetic.make_lc0_planes(300, 5)
    policy, wdl, ml = engine.evaluate(synthetic.lc0_planes_tensor(lc0))
    ref_policy, ref_wdl, ref_ml = oracle.forward(weights, synthetic.lc0_to_dense(lc0), depth=3, mode="bf16")
    torch.testing.assert_close(policy, ref_policy, atol=POLICY_ATOL, rtol=1e-2)
    assert argmax_agreement(policy, ref_policy) >= 0.995
    # The engine returns WDL probabilities (runtime.cu:309-328), not logits.
    torch.testing.assert_close(wdl, oracle.wdl_probabilities(ref_wdl), atol=WDL_PROB_ATOL, rtol=0)
    torch.testing.assert_close(ml, ref_ml, atol=POLICY_ATOL, rtol=1e-2)
    engine.close()


def test_engine_rejects_oversized_batch(tmp_path) -> None:
    from ce4b200 import Engine, export_model, synthetic

    model, _ = _dense(128, 1, seed=2)
    path = tmp_path / "small.safetensors"
    export_model(model, path)
    engine = Engine.load(path, gpu=0, max_batch=64)
    with pytest.raises(ValueError):
        engine.evaluate(synthetic.lc0_planes_tensor(synthetic.make_lc0_planes(65, 1)))
    engine.close()


@pytest.mark.parametrize("arch", ["dense", "moe64a2"])
def test_pipelined_evaluate_matches_blocking(tmp_path, arch: str) -> None:
    """Calls alternate over two streams (each call's copies overlap the other's forward
    through the model's two I/O slots); every result equals the blocking call's."""

    from ce4b200 import Engine, Moe64A2ChessNet, Moe64A2ChessNetConfig, export_model, synthetic

    if arch == "dense":
        model, _ = _dense(256, 2, seed=4)
    else:
        model = Moe64A2ChessNet(Moe64A2ChessNetConfig(d_model=128, depth=2, expansion_ratio=1.0))
        synthetic.load_into(model, synthetic.make_moe_weights(d_model=128, depth=2, expert_hidden=128, seed=4))
    path = tmp_path / f"{arch}.safetensors"
    export_model(model, path)
    engine = Engine.load(path, gpu=0, max_batch=1024)
    batches = [synthetic.lc0_planes_tensor(synthetic.make_lc0_planes(b, 40 + i)).pin_memory()
               for i, b in enumerate([1024, 1024, 640, 1024, 640, 1024])]
    expected = [engine.evaluate(p) for p in batches]
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    outs = [engine.outputs(int(p.shape[0])) for p in batches]
    for i, (p, o) in enumerate(zip(batches, outs)):
        engine.evaluate_async(p, o, streams[i % 2])
    for s in streams:
        s.synchronize()
    for (pol, wdl, ml), (epol, ewdl, eml) in zip(outs, expected):
        assert torch.equal(pol, epol)
        assert torch.equal(wdl, ewdl)
        assert torch.equal(ml, eml)
    engine.close()
