"""CPU oracle of the moe64a2 forward — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this module, as
the checker; the product path never calls it.

The reference has no runnable CPU MoE forward (its portable MoE model is a FLOP surrogate,
src/chess_engine_4/model/reference.py:104-137), so this restates the eval path of
``MoeBlock.forward`` (src/chess_engine_4/model/moe.py:160-180) with
``_run_experts_static`` (:226-287) and the expert math of the reference's custom kernels
(kernels/src/common/moe_impl.cuh:107-210; inference copy kernels/src/inference/
moe_bf16_impl.cuh:171-238):

* n = RMSNorm(x) (BF16 out); router logits = bf16(n . W_r^T) as FP32 (moe.py:162-163);
* experts = top-2 of (logits - router_qb_beta), the lower index winning ties, as the
  reference runtime's RouteKernel does (moe_bf16_impl.cuh:38-51); pinned against the
  reference's own ``_quantile_balancing_update`` in tests/golden/routing.npz;
* weights = softmax over all 64 raw logits (FP32), taken at the two experts, not
  renormalised, rounded to BF16 (moe.py:177, 261);
* per route: g, u = bf16(n . Wg_e^T), bf16(n . Wu_e^T); h = bf16(silu(g) * u);
  y = bf16((h . Wd_e^T) * p) — the probability scales the FP32 down-projection
  accumulator, as the custom and runtime kernels do (moe_impl.cuh:163-210);
* routed = bf16(y_0 + y_1) (``routed.sum(dim=1)`` on BF16, moe.py:287);
  x <- bf16(x + routed) (moe.py:180).

``mode="fp32"`` drops every BF16 rounding (the routing decision still uses BF16 logits,
because the reference's router output is BF16).
"""

from __future__ import annotations

import torch

from . import dense

EXPERTS = 64


def _bf16(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.bfloat16).to(torch.float32)


def route_top2(logits: torch.Tensor, beta: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """(experts [T,2] int64, weights [T,2] float32 before BF16 rounding).

    ``logits`` are the FP32 values of BF16 router outputs."""

    scores = logits - beta.to(torch.float32)
    # Stable descending sort: equal scores keep ascending expert order (lower index wins).
    experts = torch.sort(scores, dim=1, descending=True, stable=True).indices[:, :2]
    probs = torch.softmax(logits, dim=-1)
    return experts, probs.gather(1, experts)


def route_slots(flat_experts: torch.Tensor) -> torch.Tensor:
    """Slot of each route within its expert, in route order (moe.py:36-47 semantics)."""

    counts = torch.bincount(flat_experts, minlength=EXPERTS)
    order = torch.argsort(flat_experts, stable=True)
    starts = torch.cumsum(counts, 0) - counts
    slots = torch.empty_like(flat_experts)
    slots[order] = torch.arange(flat_experts.numel()) - starts[flat_experts[order]]
    return slots


def moe_block(
    x: torch.Tensor,
    weights: dict[str, torch.Tensor],
    layer: int,
    *,
    eps: float = 1e-6,
    mode: str = "bf16",
    forced_experts: torch.Tensor | None = None,
    record: list | None = None,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """One MoE block. Returns (x_out [T,d], experts [T,2], tokens_per_expert [64]).

    ``forced_experts`` [T,2] replaces the top-2 choice (a teacher-forced check: the weights
    are still the softmax of this block's own logits at those experts). ``record``, if
    given, receives (own top-2 choice, scores = logits - beta) of this block."""

    rnd = _bf16 if mode == "bf16" else (lambda t: t)
    p = f"blocks.{layer}"
    f = {k: v.to(torch.float32) for k, v in weights.items() if k.startswith(p + ".")}
    n = rnd(dense._rmsnorm(x, f[f"{p}.norm.weight"], eps))
    logits = _bf16(n @ f[f"{p}.router.weight"].T)
    beta = weights[f"{p}.router_qb_beta"]
    experts, probs = route_top2(logits, beta)
    if record is not None:
        record.append((experts, logits - beta.to(torch.float32)))
    if forced_experts is not None:
        experts = forced_experts.to(torch.int64)
        probs = torch.softmax(logits, dim=-1).gather(1, experts)
    probs = rnd(probs)
    gate_up = f[f"{p}.experts.gate_up.weight"]
    down = f[f"{p}.experts.down.weight"]
    h_e = down.shape[2]
    routed = torch.zeros_like(x)
    ys = torch.zeros(x.shape[0], 2, x.shape[1])
    for e in range(EXPERTS):
        for k in range(2):
            rows = (experts[:, k] == e).nonzero(as_tuple=True)[0]
            if rows.numel() == 0:
                continue
            gu = n[rows] @ gate_up[e].T
            g, u = rnd(gu[:, :h_e]), rnd(gu[:, h_e:])
            hidden = rnd(g / (1.0 + torch.exp(-g)) * u)
            ys[rows, k] = rnd((hidden @ down[e].T) * probs[rows, k : k + 1])
    routed = rnd(ys[:, 0] + ys[:, 1])
    counts = torch.bincount(experts.reshape(-1), minlength=EXPERTS)
    return rnd(x + routed), experts, counts


def forward(
    weights: dict[str, torch.Tensor],
    planes: torch.Tensor,
    *,
    depth: int,
    history_length: int = 8,
    eps: float = 1e-6,
    mode: str = "bf16",
    forced_experts: torch.Tensor | None = None,
    record: list | None = None,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """moe64a2 tower: even layers MoE, odd layers dense (moe.py:354-366).

    ``forced_experts`` [depth/2, B, 2] teacher-forces every MoE layer's expert choice;
    ``record`` collects each MoE layer's own (top-2 choice, scores) (see moe_block).
    Returns (policy [B,1858], wdl [B,3], moves_left [B], tokens_per_expert [depth/2, 64])."""

    counts: list[torch.Tensor] = []

    def moe_forward(x: torch.Tensor, layer: int, m: str) -> torch.Tensor:
        forced = forced_experts[layer // 2] if forced_experts is not None else None
        out, _, c = moe_block(x, weights, layer, eps=eps, mode=m, forced_experts=forced, record=record)
        counts.append(c)
        return out

    policy, wdl, ml = dense.forward(
        weights,
        planes,
        depth=depth,
        history_length=history_length,
        eps=eps,
        mode=mode,
        moe_layers=frozenset(range(0, depth, 2)),
        moe_forward=moe_forward,
    )
    return policy, wdl, ml, torch.stack(counts)
