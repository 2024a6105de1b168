"""Generate the golden fixtures in this directory from the reference implementation.

Run in a container that has the reference source tree (read-only is fine):

    python tests/golden/make_golden.py --reference /path/to/chess-engine-4/src

Each dense fixture runs the reference's own portable model, ``PortableChessNet``
(src/chess_engine_4/model/reference.py:60-101), in FP32 on seeded synthetic weights and
planes, and stores its outputs with the seeds and a weight checksum; one more runs it
moved to BF16. The MXFP8 fixture holds the codes and swizzled scales that the reference's
own torch quantiser (torch_mxfp8_quantize and scale_swizzle in
third_party/ThunderKittens/kernels/gemm/mxfp8_b200/test_quantize.py, lifted out of the file
with ``ast``) gives for a seeded sample. The routing fixture
stores outputs of the reference's ``_quantile_balancing_update`` and ``_route_slots``
(src/chess_engine_4/model/moe.py:36-71) plus the reference tests' known answers
(tests/test_model_and_losses.py:215-220, 230-236). The fixtures are small; the tests
regenerate the weights from the seeds and check the checksum first.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO / "chess-engine-4_b200"))

from ce4b200 import synthetic  # noqa: E402

DENSE_CASES = [
    # name, d_model, depth, expansion_ratio, history_length, batch, weight seed, plane seed
    ("dense_d64_l2_r2", 64, 2, 2.0, 8, 8, 11, 12),
    ("dense_d128_l6_r3", 128, 6, 3.0, 8, 8, 0, 1),
    ("dense_d64_l1_r2_h2", 64, 1, 2.0, 2, 4, 21, 22),
]


def weight_checksum(weights: dict[str, torch.Tensor]) -> str:
    h = hashlib.sha256()
    for name in sorted(weights):
        h.update(name.encode())
        h.update(weights[name].contiguous().view(torch.uint8).numpy().tobytes())
    return h.hexdigest()


def portable_state(weights: dict[str, torch.Tensor], depth: int) -> dict[str, torch.Tensor]:
    """Safetensors names -> PortableChessNet names; heads sliced 1888->1858, 32->3, 32->1."""

    f = {k: v.to(torch.float32) for k, v in weights.items()}
    s = {
        "input.weight": f["input.weight"],
        "input.bias": f["input.bias"],
        "norm.weight": f["final_norm.weight"],
        "policy_head.weight": f["policy.weight"][:1858],
        "policy_head.bias": f["policy.bias"][:1858],
        "wdl_head.weight": f["wdl.weight"][:3],
        "wdl_head.bias": f["wdl.bias"][:3],
        "moves_left_head.weight": f["moves_left.weight"][:1],
        "moves_left_head.bias": f["moves_left.bias"][:1],
    }
    for layer in range(depth):
        p = f"blocks.{layer}"
        s[f"{p}.norm.weight"] = f[f"{p}.norm.weight"]
        s[f"{p}.gate_up.weight"] = f[f"{p}.gate_up.weight"]
        s[f"{p}.down.weight"] = f[f"{p}.down.weight"]
    return s


def dense_fixture(name, d, depth, ratio, hist, batch, wseed, pseed) -> None:
    from chess_engine_4.model.dense import DenseChessNetConfig
    from chess_engine_4.model.reference import PortableChessNet

    hidden = int(d * ratio)
    weights = synthetic.make_dense_weights(
        d_model=d, depth=depth, hidden_dim=hidden, seed=wseed, history_length=hist
    )
    lc0 = synthetic.make_lc0_planes(batch, pseed)
    planes = synthetic.lc0_to_dense(lc0)
    model = PortableChessNet(
        DenseChessNetConfig(d_model=d, depth=depth, expansion_ratio=ratio, history_length=hist)
    )
    model.load_state_dict(portable_state(weights, depth))
    with torch.no_grad():
        out = model(planes.clone())
    np.savez_compressed(
        HERE / f"{name}.npz",
        policy=out.policy_logits.numpy().astype(np.float32),
        wdl=out.wdl_logits.numpy().astype(np.float32),
        moves_left=out.moves_left.numpy().astype(np.float32),
        meta=np.array(
            json.dumps(
                {
                    "d_model": d,
                    "depth": depth,
                    "expansion_ratio": ratio,
                    "history_length": hist,
                    "batch": batch,
                    "weight_seed": wseed,
                    "plane_seed": pseed,
                    "weight_sha256": weight_checksum(weights),
                    "generator": "ce4b200.synthetic.make_dense_weights / make_lc0_planes",
                    "reference": "chess_engine_4.model.reference.PortableChessNet (fp32)",
                }
            )
        ),
    )


def dense_bf16_fixture() -> None:
    """PortableChessNet moved to BF16 (weights cast once, BF16 planes), on the
    dense_d128_l6_r3 weights: pins the CPU baseline's BF16 arm (oracle.dense.PortableForward
    with dtype=bfloat16) to the reference module's own BF16 forward."""
    from chess_engine_4.model.dense import DenseChessNetConfig
    from chess_engine_4.model.reference import PortableChessNet

    name, d, depth, ratio, hist, batch, wseed, pseed = DENSE_CASES[1]
    weights = synthetic.make_dense_weights(
        d_model=d, depth=depth, hidden_dim=int(d * ratio), seed=wseed, history_length=hist
    )
    planes = synthetic.lc0_to_dense(synthetic.make_lc0_planes(batch, pseed)).to(torch.bfloat16)
    model = PortableChessNet(
        DenseChessNetConfig(d_model=d, depth=depth, expansion_ratio=ratio, history_length=hist)
    )
    model.load_state_dict(portable_state(weights, depth))
    model = model.to(torch.bfloat16)
    with torch.no_grad():
        out = model(planes.clone())
    np.savez_compressed(
        HERE / f"{name}_bf16module.npz",
        policy=out.policy_logits.float().numpy(),
        wdl=out.wdl_logits.float().numpy(),
        moves_left=out.moves_left.float().numpy(),
        meta=np.array(json.dumps({
            "d_model": d, "depth": depth, "expansion_ratio": ratio, "history_length": hist,
            "batch": batch, "weight_seed": wseed, "plane_seed": pseed,
            "weight_sha256": weight_checksum(weights),
            "reference": "chess_engine_4.model.reference.PortableChessNet.to(torch.bfloat16), BF16 planes",
        })),
    )


MXFP8_SOURCE = "third_party/ThunderKittens/kernels/gemm/mxfp8_b200/test_quantize.py"


def reference_mxfp8_functions(reference_root: Path) -> dict:
    """``torch_mxfp8_quantize`` and ``scale_swizzle`` from the reference's quantiser test
    (MXFP8_SOURCE), taken out of the file with ``ast`` and compiled on their own: the module
    itself imports the compiled ``_C`` extension, which is not built here."""
    import ast

    path = reference_root / MXFP8_SOURCE
    tree = ast.parse(path.read_text(), filename=str(path))
    wanted = {"torch_mxfp8_quantize", "scale_swizzle"}
    body = [n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name in wanted]
    assert {n.name for n in body} == wanted, "reference quantiser functions not found"
    namespace: dict = {"torch": torch}
    exec(compile(ast.Module(body=body, type_ignores=[]), str(path), "exec"), namespace)
    return namespace


def mxfp8_sample(seed: int = 31, rows: int = 256, cols: int = 256) -> torch.Tensor:
    """BF16 test matrix: per-row magnitudes over ~24 binades, 5 % exact zeros, values near
    powers of two, and one all-zero 32-block (row 5, columns 64..95)."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, cols, generator=g) * torch.exp2(torch.randint(-12, 12, (rows, 1), generator=g).float())
    x[torch.rand(rows, cols, generator=g) < 0.05] = 0
    x[9, :32] = torch.exp2(torch.randint(-4, 4, (32,), generator=g).float())  # exact powers of two
    x[10, :32] = 448.0 * torch.exp2(torch.randint(-6, 6, (32,), generator=g).float())
    x[5, 64:96] = 0
    return x.bfloat16()


def mxfp8_fixture(reference_root: Path) -> None:
    fns = reference_mxfp8_functions(reference_root)
    x = mxfp8_sample()
    codes, scales = fns["torch_mxfp8_quantize"](x)
    np.savez_compressed(
        HERE / "mxfp8_reference_quantizer.npz",
        codes=codes.view(torch.uint8).numpy(),
        scales=fns["scale_swizzle"](scales).numpy(),
        meta=np.array(json.dumps({
            "sample": "tests/golden/make_golden.py:mxfp8_sample(seed=31, rows=256, cols=256)",
            "input_sha256": hashlib.sha256(x.view(torch.int16).numpy().tobytes()).hexdigest(),
            "reference": MXFP8_SOURCE + ": torch_mxfp8_quantize, scale_swizzle",
        })),
    )


def routing_fixture() -> None:
    from chess_engine_4.model.moe import (
        _quantile_balancing_update,
        _route_slots,
        moe64a2_parameter_count,
    )

    g = torch.Generator().manual_seed(5)
    # BF16-valued logits (the router output is BF16) and a Zipf-skewed fp32 beta.
    logits = (torch.randn(256, 64, generator=g) * 0.5).to(torch.bfloat16).to(torch.float32)
    beta = synthetic.zipf_router_bias(7)
    indices, _ = _quantile_balancing_update(logits, topk=2, beta=beta, update_beta=False)
    flat = indices.reshape(-1)
    counts = torch.bincount(flat, minlength=64)
    slots = _route_slots(flat, counts)
    kat_slots = _route_slots(torch.tensor([2, 0, 2, 1, 0, 2]), torch.tensor([2, 1, 3]))
    np.savez_compressed(
        HERE / "routing.npz",
        logits=logits.numpy(),
        beta=beta.numpy(),
        indices=indices.numpy().astype(np.int64),
        slots=slots.numpy().astype(np.int64),
        counts=counts.numpy().astype(np.int64),
        kat_slots=kat_slots.numpy().astype(np.int64),
        kat_param_count=np.array(moe64a2_parameter_count(d_model=64, depth=2, expansion_ratio=2.0)),
    )


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", required=True, help="path to the reference src/ directory")
    args = parser.parse_args()
    sys.path.insert(0, args.reference)
    torch.manual_seed(0)
    for case in DENSE_CASES:
        dense_fixture(*case)
    dense_bf16_fixture()
    mxfp8_fixture(Path(args.reference).resolve().parent)
    routing_fixture()
    print("wrote fixtures to", HERE)


if __name__ == "__main__":
    main()
