"""Pins the CPU oracle to outputs of the reference implementation itself.

The fixtures in tests/golden/ were produced by tests/golden/make_golden.py, which runs the
reference's portable model (``PortableChessNet``) and its routing helpers on seeded
inputs. The weights are regenerated here from the recorded seeds (checked by SHA-256)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import load_golden

DENSE_FIXTURES = ["dense_d64_l2_r2", "dense_d128_l6_r3", "dense_d64_l1_r2_h2"]


@pytest.mark.parametrize("name", DENSE_FIXTURES)
def test_dense_oracle_reproduces_reference(name: str) -> None:
    from ce4b200 import synthetic
    from oracle import dense as oracle
    from tests_golden_util import weight_checksum

    meta, data = load_golden(name)
    weights = synthetic.make_dense_weights(
        d_model=meta["d_model"],
        depth=meta["depth"],
        hidden_dim=int(meta["d_model"] * meta["expansion_ratio"]),
        seed=meta["weight_seed"],
        history_length=meta["history_length"],
    )
    assert weight_checksum(weights) == meta["weight_sha256"], "weight generator drifted"
    planes = synthetic.lc0_to_dense(synthetic.make_lc0_planes(meta["batch"], meta["plane_seed"]))
    policy, wdl, moves_left = oracle.forward(
        weights, planes, depth=meta["depth"], history_length=meta["history_length"], mode="fp32"
    )
    torch.testing.assert_close(policy, torch.from_numpy(data["policy"]), atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(wdl, torch.from_numpy(data["wdl"]), atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(moves_left, torch.from_numpy(data["moves_left"]), atol=1e-5, rtol=1e-5)


def test_bf16_oracle_stays_near_fp32() -> None:
    from ce4b200 import synthetic
    from oracle import dense as oracle

    meta, _ = load_golden("dense_d128_l6_r3")
    weights = synthetic.make_dense_weights(
        d_model=128, depth=6, hidden_dim=384, seed=meta["weight_seed"]
    )
    planes = synthetic.lc0_to_dense(synthetic.make_lc0_planes(64, 3))
    p32 = oracle.forward(weights, planes, depth=6, mode="fp32")[0]
    p16 = oracle.forward(weights, planes, depth=6, mode="bf16")[0]
    assert (p16 - p32).abs().max() < 2e-2


def test_oracle_does_not_modify_planes() -> None:
    from ce4b200 import synthetic
    from oracle import dense as oracle

    weights = synthetic.make_dense_weights(d_model=64, depth=1, hidden_dim=128, seed=1)
    planes = synthetic.lc0_to_dense(synthetic.make_lc0_planes(2, 2))
    before = planes.clone()
    oracle.forward(weights, planes, depth=1)
    assert torch.equal(planes, before)


def test_input_formats_round_trip() -> None:
    """lc0 records, dense planes and the bit-packed layout describe the same input."""

    from ce4b200 import synthetic

    lc0 = synthetic.make_lc0_planes(5, 4, aux_constant=True)
    dense = synthetic.lc0_to_dense(lc0)
    packed, scalars = synthetic.lc0_to_packed(lc0)
    # Expand the packed layout the way PlaneInputExpander does (MSB first per byte).
    bits = np.unpackbits(packed.numpy(), axis=-1, bitorder="big").reshape(5, 104, 8, 8)
    expanded = np.concatenate(
        [bits.astype(np.float32), np.broadcast_to(scalars.numpy()[:, :, None, None], (5, 8, 8, 8))],
        axis=1,
    )
    np.testing.assert_array_equal(expanded, dense.numpy())
    assert dense[:, 109].unique().numel() <= 5  # one rule-50 value per position
    assert torch.all(dense[:, 111] == 1)


def test_route_slots_known_answer_and_routing_fixture() -> None:
    _, data = load_golden("routing")
    np.testing.assert_array_equal(data["kat_slots"], np.array([0, 0, 1, 0, 1, 2]))
    assert int(data["kat_param_count"]) == 2_212_000
    # Top-2 of (logit - beta) with the lower index winning ties reproduces the reference.
    logits = torch.from_numpy(data["logits"])
    beta = torch.from_numpy(data["beta"])
    scores = logits - beta
    order = torch.sort(scores, dim=1, descending=True, stable=True).indices[:, :2]
    np.testing.assert_array_equal(order.numpy(), data["indices"])
