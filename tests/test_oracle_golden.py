"""Pins the CPU oracle to outputs of the reference implementation itself.

The fixtures in tests/golden/ were produced by tests/golden/make_golden.py, which runs the
reference's portable model (``PortableChessNet``) and its routing helpers on seeded
inputs. The weights are regenerated here from the recorded seeds (checked by SHA-256)."""

from __future__ import annotations

from pathlib import Path

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


def test_portable_forward_reproduces_reference_module_in_fp32_and_bf16() -> None:
    """oracle.dense.PortableForward (the CPU baseline's implementation) reproduces the
    reference's PortableChessNet bit for bit: in FP32, and moved to BF16."""
    from ce4b200 import synthetic
    from oracle import dense as oracle

    for name, dtype in (("dense_d128_l6_r3", torch.float32), ("dense_d128_l6_r3_bf16module", torch.bfloat16)):
        meta, data = load_golden(name)
        weights = synthetic.make_dense_weights(
            d_model=meta["d_model"], depth=meta["depth"],
            hidden_dim=int(meta["d_model"] * meta["expansion_ratio"]), seed=meta["weight_seed"],
        )
        planes = synthetic.lc0_to_dense(synthetic.make_lc0_planes(meta["batch"], meta["plane_seed"])).to(dtype)
        with torch.no_grad():
            policy, wdl, ml = oracle.PortableForward(weights, depth=meta["depth"], dtype=dtype)(planes)
        assert torch.equal(policy.float(), torch.from_numpy(data["policy"])), name
        assert torch.equal(wdl.float(), torch.from_numpy(data["wdl"])), name
        assert torch.equal(ml.float(), torch.from_numpy(data["moves_left"])), name


def test_mxfp8_oracle_matches_reference_quantizer() -> None:
    """oracle/mxfp8.c against codes and scales that the reference's own torch quantiser
    produced (tests/golden/make_golden.py runs torch_mxfp8_quantize and scale_swizzle from
    the reference's test_quantize.py). Every E4M3 code and every scale of a non-zero block
    is identical. An all-zero block is the one documented difference: the reference's
    kernel clamps the scale at 1e-12 (E8M0 code 88), which oracle/mxfp8.c and the GPU
    quantiser follow, while the torch restatement clamps the exponent at -127 (code 0)."""
    import hashlib
    import sys

    from oracle import mxfp8

    sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
    from make_golden import mxfp8_sample

    meta, data = load_golden("mxfp8_reference_quantizer")
    x = mxfp8_sample()
    assert hashlib.sha256(x.view(torch.int16).numpy().tobytes()).hexdigest() == meta["input_sha256"]
    codes, scales = mxfp8.quantize(x)
    assert torch.equal(codes, torch.from_numpy(data["codes"]))
    ours = mxfp8.unswizzle_scales(scales)
    ref = mxfp8.unswizzle_scales(torch.from_numpy(data["scales"]))
    zero_block = x.float().abs().view(x.shape[0], -1, 32).amax(-1) == 0
    assert int(zero_block.sum()) == 1
    assert torch.equal(ours[~zero_block], ref[~zero_block])
    assert torch.all(ours[zero_block] == 88) and torch.all(ref[zero_block] == 0)
