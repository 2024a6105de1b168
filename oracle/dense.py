"""CPU oracle of the dense forward — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use this module, as
the checker; the product path (libce4b200) never calls it.

Two restatements of the reference's dense tower on the same Safetensors-named weights:

* ``mode="fp32"``: the reference's portable PyTorch model, ``PortableChessNet``
  (src/chess_engine_4/model/reference.py:60-101, _DenseBlock :17-43), computed in FP32
  with the BF16 weights upcast. History selection and the rule-50 / 99 normalisation
  follow src/chess_engine_4/model/dense.py:34-51, 188-199. Pinned against outputs of the
  reference itself (tests/golden/make_golden.py).
* ``mode="bf16"``: the same network with the BF16 rounding points of the reference's
  deployed forward (kernels/src/inference/runtime.cu:182-336, 578-645; TE's fused-bias
  Linear for the input and head projections): inputs rounded to BF16; every GEMM
  accumulates in FP32 and rounds its output to BF16; RMSNorm computes in FP32 and rounds
  once; SwiGLU rounds gate and up, then the product; the residual add rounds the sum;
  head logits are bf16(acc + bias).
"""

from __future__ import annotations

import torch

POLICY_SIZE = 1858
HISTORY_PLANES = 104
PLANES_PER_HISTORY = 13


def _bf16(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.bfloat16).to(torch.float32)


def select_and_normalize(planes: torch.Tensor, history_length: int) -> torch.Tensor:
    """[B,112,8,8] -> [B, sel*64] float32 (dense.py:45-51 history select, :34-42 rule-50/99).
    Does not modify ``planes``."""

    x = planes.to(torch.float32)
    hp = history_length * PLANES_PER_HISTORY
    if hp != HISTORY_PLANES:
        x = torch.cat((x[:, :hp], x[:, HISTORY_PLANES:]), dim=1)
    else:
        x = x.clone()
    x[:, hp + 5] = x[:, hp + 5] / 99.0
    return x.flatten(start_dim=1)


def mx_dequant(t: torch.Tensor) -> torch.Tensor:
    """MXFP8 round trip of a BF16-valued matrix (quantise with the C restatement of the
    reference's recipe, oracle/mxfp8.c, then dequantise); rows are padded to 128."""

    from . import mxfp8

    rows, cols = t.shape
    pad = (-rows) % 128
    tb = torch.cat([t, t.new_zeros(pad, cols)]) if pad else t
    codes, scales = mxfp8.quantize(tb.to(torch.bfloat16))
    return mxfp8.dequantize(codes, scales)[:rows]


def _rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    inv = torch.rsqrt(x.pow(2).mean(dim=-1, keepdim=True) + eps)
    return x * inv * w


def forward(
    weights: dict[str, torch.Tensor],
    planes: torch.Tensor,
    *,
    depth: int,
    history_length: int = 8,
    eps: float = 1e-6,
    mode: str = "fp32",
    moe_layers: frozenset[int] = frozenset(),
    moe_forward=None,
    fold_norm: bool = False,
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Returns (policy_logits [B,1858], wdl_logits [B,3], moves_left [B]) in float32.

    ``moe_layers`` / ``moe_forward`` let oracle.moe reuse this tower for moe64a2.

    ``fold_norm`` (bf16 mode, dense only) restates the arithmetic of libce4b200's
    persistent dense forward instead of the reference's rounding points: each RMSNorm
    weight is folded into the next linear's weight, W' = bf16(W * diag(w)), and the row
    scale r = rsqrt(mean(x^2) + eps) multiplies the FP32 product, so the normalised row
    is never rounded: gate/up = bf16(r * (x W'^T)), heads = bf16(r * (x W'_h^T) + b)."""

    if mode not in ("fp32", "bf16", "mxfp8"):
        raise ValueError(mode)
    if fold_norm and (mode != "bf16" or moe_layers):
        raise ValueError("fold_norm restates the dense BF16 persistent forward only")
    rnd = _bf16 if mode in ("bf16", "mxfp8") else (lambda t: t)
    # MXFP8 (all linears, recipe of the reference's custom path): both GEMM operands are
    # MXFP8 round trips of their BF16 values; everything else is the BF16 forward.
    q = mx_dequant if mode == "mxfp8" else (lambda t: t)
    f = {k: v.to(torch.float32) for k, v in weights.items()}
    a = rnd(select_and_normalize(planes, history_length))
    x = rnd(q(a) @ q(f["input.weight"]).T + f["input.bias"])
    for layer in range(depth):
        p = f"blocks.{layer}"
        if layer in moe_layers:
            assert moe_forward is not None
            x = moe_forward(x, layer, mode)
            continue
        if fold_norm:
            r = torch.rsqrt(x.pow(2).mean(dim=-1, keepdim=True) + eps)
            gu = (x @ _bf16(f[f"{p}.gate_up.weight"] * f[f"{p}.norm.weight"]).T) * r
        else:
            n = rnd(_rmsnorm(x, f[f"{p}.norm.weight"], eps))
            gu = q(n) @ q(f[f"{p}.gate_up.weight"]).T
        h = gu.shape[1] // 2
        g, u = rnd(gu[:, :h]), rnd(gu[:, h:])
        hidden = rnd(g / (1.0 + torch.exp(-g)) * u)
        x = rnd(x + rnd(q(hidden) @ q(f[f"{p}.down.weight"]).T))
    heads = torch.cat([f["policy.weight"], f["wdl.weight"], f["moves_left.weight"]])
    if fold_norm:
        r = torch.rsqrt(x.pow(2).mean(dim=-1, keepdim=True) + eps)
        logits = (x @ _bf16(heads * f["final_norm.weight"]).T) * r
    else:
        n = q(rnd(_rmsnorm(x, f["final_norm.weight"], eps)))
        logits = n @ q(heads).T
    ps = f["policy.weight"].shape[0]
    policy = rnd(logits[:, :POLICY_SIZE] + f["policy.bias"][:POLICY_SIZE])
    wdl = rnd(logits[:, ps : ps + 3] + f["wdl.bias"][:3])
    moves_left = rnd(logits[:, ps + 32 : ps + 33] + f["moves_left.bias"][:1])[:, 0]
    return policy, wdl, moves_left


class PortableForward:
    """``PortableChessNet`` (src/chess_engine_4/model/reference.py:60-101) restated as a
    function of Safetensors-named weights that are cast to ``dtype`` once, as the module is
    when it is moved to that dtype; ``forward`` then runs the module's own operations in
    that dtype: history select and rule-50 / 99 (dense.py:34-51), ``Linear`` with bias,
    per block ``x + down(silu(gate) * up)`` over ``RMSNorm(x)`` (reference.py:17-43), final
    ``RMSNorm`` and the three heads (1858 / 3 / 1 columns of the stored 1888 / 32 / 32).
    With ``dtype=torch.float32`` this is ``forward(mode="fp32")``; with ``torch.bfloat16`` it
    is the reference module run in BF16 on the CPU (the CPU baseline's BF16 arm), pinned to
    the reference's own BF16 output in tests/golden/."""

    def __init__(self, weights: dict[str, torch.Tensor], *, depth: int, history_length: int = 8,
                 eps: float = 1e-6, dtype: torch.dtype = torch.float32) -> None:
        self.depth, self.history_length, self.eps, self.dtype = depth, history_length, eps, dtype
        c = {k: v.detach().to(dtype).contiguous() for k, v in weights.items()}
        self.w = c
        self.heads = {
            "policy": (c["policy.weight"][:POLICY_SIZE].contiguous(), c["policy.bias"][:POLICY_SIZE].contiguous()),
            "wdl": (c["wdl.weight"][:3].contiguous(), c["wdl.bias"][:3].contiguous()),
            "moves_left": (c["moves_left.weight"][:1].contiguous(), c["moves_left.bias"][:1].contiguous()),
        }

    def __call__(self, planes: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        from torch.nn import functional as F

        w, d = self.w, self.w["input.weight"].shape[0]
        x = planes.to(self.dtype)
        hp = self.history_length * PLANES_PER_HISTORY
        x = torch.cat((x[:, :hp], x[:, HISTORY_PLANES:]), dim=1) if hp != HISTORY_PLANES else x.clone()
        x[:, hp + 5] = x[:, hp + 5] / 99.0
        x = F.linear(x.flatten(start_dim=1), w["input.weight"], w["input.bias"])
        for layer in range(self.depth):
            p = f"blocks.{layer}"
            n = F.rms_norm(x, (d,), w[f"{p}.norm.weight"], self.eps)
            gate, up = F.linear(n, w[f"{p}.gate_up.weight"]).chunk(2, dim=-1)
            x = x + F.linear(F.silu(gate) * up, w[f"{p}.down.weight"])
        x = F.rms_norm(x, (d,), w["final_norm.weight"], self.eps)
        policy = F.linear(x, *self.heads["policy"])
        wdl = F.linear(x, *self.heads["wdl"])
        moves_left = F.linear(x, *self.heads["moves_left"]).squeeze(-1)
        return policy, wdl, moves_left


def wdl_probabilities(wdl_logits: torch.Tensor) -> torch.Tensor:
    """FP32 softmax of the three logits (kernels/src/inference/runtime.cu:309-328)."""

    return torch.softmax(wdl_logits.to(torch.float32), dim=-1)
