"""Seeded synthetic inputs and weights with the shapes and value distributions of the
benchmark configurations (no public dataset or checkpoint is used).

Planes: 112 lc0 planes per position. Planes 0-107 are Bernoulli(p) bit masks with
value 1; plane 108 (en passant) is empty; plane 109 (rule-50 ply) covers the board with
an integer in [0, 99]; plane 110 is empty; plane 111 is all ones. With
``aux_constant=True`` the aux planes 104-107 are full-board 0/1 constants instead, which
the bit-packed training layout can represent.

Weights: BF16 N(0, std) for every matrix, Safetensors v1 names. RMSNorm weights are 1 +
N(0, norm_std) and biases N(0, bias_std). MoE routers are N(0, std); the quantile-balancing
offset of expert e is ``-0.1 * z_e / mean(z)`` with ``z`` Zipf(s) weights over a seeded
permutation of the experts, which skews the top-2 load toward a few experts.
"""

from __future__ import annotations

import numpy as np
import torch

INPUT_PLANES = 112
HISTORY_PLANES = 104
POLICY_SIZE = 1858
POLICY_STORAGE = 1888
EXPERTS = 64

LC0_PLANE_DTYPE = np.dtype([("mask", "<u8"), ("value", "<f4"), ("reserved", "<u4")])


def _generator(seed: int, device: str | torch.device = "cpu") -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def make_lc0_planes(
    batch: int, seed: int, *, density: float = 0.08, aux_constant: bool = False
) -> np.ndarray:
    """Structured array ``[B, 112]`` of ``InputPlane{u64 mask, f32 value}`` records."""

    g = _generator(seed)
    bits = torch.rand(batch, INPUT_PLANES, 64, generator=g) < density
    values = torch.ones(batch, INPUT_PLANES)
    if aux_constant:
        on = torch.rand(batch, 4, generator=g) < 0.5
        bits[:, 104:108] = on[:, :, None]
    bits[:, 108] = False
    bits[:, 109] = True
    values[:, 109] = torch.randint(0, 100, (batch,), generator=g).float()
    bits[:, 110] = False
    bits[:, 111] = True
    packed = np.packbits(bits.numpy().astype(np.uint8), axis=-1, bitorder="little")
    masks = packed.reshape(batch, INPUT_PLANES, 8).view("<u8").reshape(batch, INPUT_PLANES)
    out = np.zeros((batch, INPUT_PLANES), dtype=LC0_PLANE_DTYPE)
    out["mask"] = masks
    out["value"] = values.numpy()
    return out


def lc0_to_dense(planes: np.ndarray) -> torch.Tensor:
    """``[B, 112, 8, 8]`` float32 planes (square s = rank*8 + file = bit s of the mask)."""

    masks = np.ascontiguousarray(planes["mask"]).view(np.uint8).reshape(-1, INPUT_PLANES, 8)
    bits = np.unpackbits(masks, axis=-1, bitorder="little").reshape(-1, INPUT_PLANES, 64)
    dense = bits.astype(np.float32) * planes["value"][:, :, None]
    return torch.from_numpy(dense.reshape(-1, INPUT_PLANES, 8, 8).copy())


def lc0_to_packed(planes: np.ndarray) -> tuple[torch.Tensor, torch.Tensor]:
    """Bit-packed training layout: u8 ``[B, 104, 8]`` (byte r holds squares r*8..r*8+7,
    most significant bit first) and float32 ``[B, 8]`` aux-plane scalars. The aux planes
    must be full-board constants (``aux_constant=True``)."""

    dense = lc0_to_dense(planes).numpy()
    history = dense[:, :HISTORY_PLANES].reshape(-1, HISTORY_PLANES, 8, 8) != 0
    packed = np.packbits(history.astype(np.uint8), axis=-1, bitorder="big").reshape(
        -1, HISTORY_PLANES, 8
    )
    aux = dense[:, HISTORY_PLANES:].reshape(-1, INPUT_PLANES - HISTORY_PLANES, 64)
    if not np.all(aux == aux[:, :, :1]):
        raise ValueError("aux planes are not board constants; use aux_constant=True")
    return torch.from_numpy(packed.copy()), torch.from_numpy(aux[:, :, 0].copy())


def lc0_planes_tensor(planes: np.ndarray) -> torch.Tensor:
    """int64 ``[B, 112, 2]`` view of the 16-byte records (for ``forward_lc0``)."""

    raw = np.ascontiguousarray(planes).view(np.int64).reshape(-1, INPUT_PLANES, 2)
    return torch.from_numpy(raw.copy())


def _randn(shape: tuple[int, ...], std: float, g: torch.Generator, device: str) -> torch.Tensor:
    return (torch.randn(shape, generator=g, device=device) * std).to(torch.bfloat16)


def make_dense_weights(
    *,
    d_model: int,
    depth: int,
    hidden_dim: int,
    seed: int,
    history_length: int = 8,
    std: float = 0.02,
    norm_std: float = 0.1,
    bias_std: float = 0.02,
    device: str = "cpu",
) -> dict[str, torch.Tensor]:
    """Dense tower weights under Safetensors v1 names (BF16)."""

    g = _generator(seed, device)
    in_dim = (history_length * 13 + 8) * 64
    w: dict[str, torch.Tensor] = {}
    w["input.weight"] = _randn((d_model, in_dim), std, g, device)
    w["input.bias"] = _randn((d_model,), bias_std, g, device)
    for layer in range(depth):
        p = f"blocks.{layer}"
        w[f"{p}.norm.weight"] = (1.0 + torch.randn(d_model, generator=g, device=device) * norm_std).to(
            torch.bfloat16
        )
        w[f"{p}.gate_up.weight"] = _randn((2 * hidden_dim, d_model), std, g, device)
        w[f"{p}.down.weight"] = _randn((d_model, hidden_dim), std, g, device)
    _heads(w, d_model, std, norm_std, bias_std, g, device)
    return w


def _heads(
    w: dict[str, torch.Tensor],
    d_model: int,
    std: float,
    norm_std: float,
    bias_std: float,
    g: torch.Generator,
    device: str,
) -> None:
    w["final_norm.weight"] = (1.0 + torch.randn(d_model, generator=g, device=device) * norm_std).to(
        torch.bfloat16
    )
    w["policy.weight"] = _randn((POLICY_STORAGE, d_model), std, g, device)
    w["policy.bias"] = _randn((POLICY_STORAGE,), bias_std, g, device)
    w["wdl.weight"] = _randn((32, d_model), std, g, device)
    w["wdl.bias"] = _randn((32,), bias_std, g, device)
    w["moves_left.weight"] = _randn((32, d_model), std, g, device)
    w["moves_left.bias"] = _randn((32,), bias_std, g, device)


def zipf_router_bias(seed: int, *, s: float = 1.1, scale: float = 0.1) -> torch.Tensor:
    """``router_qb_beta`` favouring a Zipf-ranked subset of experts (beta = -bias)."""

    g = _generator(seed)
    ranks = torch.randperm(EXPERTS, generator=g) + 1
    z = 1.0 / ranks.double() ** s
    bias = scale * z / z.mean()
    return (-bias).float()


def make_moe_weights(
    *,
    d_model: int,
    depth: int,
    expert_hidden: int,
    seed: int,
    history_length: int = 8,
    std: float = 0.02,
    norm_std: float = 0.1,
    bias_std: float = 0.02,
    zipf_s: float = 1.1,
    device: str = "cpu",
) -> dict[str, torch.Tensor]:
    """moe64a2 weights under Safetensors v1 names: even layers MoE, odd layers dense 4d."""

    if depth % 2:
        raise ValueError("moe64a2 depth must be even")
    g = _generator(seed, device)
    in_dim = (history_length * 13 + 8) * 64
    w: dict[str, torch.Tensor] = {}
    w["input.weight"] = _randn((d_model, in_dim), std, g, device)
    w["input.bias"] = _randn((d_model,), bias_std, g, device)
    for layer in range(depth):
        p = f"blocks.{layer}"
        w[f"{p}.norm.weight"] = (1.0 + torch.randn(d_model, generator=g, device=device) * norm_std).to(
            torch.bfloat16
        )
        if layer % 2 == 0:
            w[f"{p}.router.weight"] = _randn((EXPERTS, d_model), std, g, device)
            w[f"{p}.router_qb_beta"] = zipf_router_bias(seed * 1000 + layer, s=zipf_s).to(device)
            w[f"{p}.experts.gate_up.weight"] = _randn(
                (EXPERTS, 2 * expert_hidden, d_model), std, g, device
            )
            w[f"{p}.experts.down.weight"] = _randn((EXPERTS, d_model, expert_hidden), std, g, device)
        else:
            w[f"{p}.gate_up.weight"] = _randn((8 * d_model, d_model), std, g, device)
            w[f"{p}.down.weight"] = _randn((d_model, 4 * d_model), std, g, device)
    _heads(w, d_model, std, norm_std, bias_std, g, device)
    return w


def load_into(model: torch.nn.Module, weights: dict[str, torch.Tensor]) -> None:
    """Copy Safetensors-named weights into a ``DenseChessNet`` / ``Moe64A2ChessNet``
    (inverse of the name mapping in src/chess_engine_4/release/export.py:164-188)."""

    from .model import DenseBlock, GroupedLinear, MoeBlock

    def put(param: torch.Tensor, value: torch.Tensor) -> None:
        with torch.no_grad():
            if param.shape != value.shape:
                raise ValueError(f"shape mismatch {tuple(param.shape)} vs {tuple(value.shape)}")
            param.copy_(value.to(param.device))

    m = model
    put(m.input.weight, weights["input.weight"])
    put(m.input.bias, weights["input.bias"])
    put(m.norm.weight, weights["final_norm.weight"])
    put(m.policy_head.weight, weights["policy.weight"])
    put(m.policy_head.bias, weights["policy.bias"])
    put(m.wdl_head.weight, weights["wdl.weight"])
    put(m.wdl_head.bias, weights["wdl.bias"])
    put(m.moves_left_head.weight, weights["moves_left.weight"])
    put(m.moves_left_head.bias, weights["moves_left.bias"])
    for i, block in enumerate(m.blocks):
        p = f"blocks.{i}"
        if isinstance(block, MoeBlock):
            put(block.norm.weight, weights[f"{p}.norm.weight"])
            put(block.router.weight, weights[f"{p}.router.weight"])
            put(block.router_qb_beta, weights[f"{p}.router_qb_beta"])
            gate_up = block.experts[0]
            down = block.experts[2]
            assert isinstance(gate_up, GroupedLinear) and isinstance(down, GroupedLinear)
            for e in range(EXPERTS):
                put(getattr(gate_up, f"weight{e}"), weights[f"{p}.experts.gate_up.weight"][e])
                put(getattr(down, f"weight{e}"), weights[f"{p}.experts.down.weight"][e])
        else:
            assert isinstance(block, DenseBlock)
            put(block.layer.layer_norm_weight, weights[f"{p}.norm.weight"])
            put(block.layer.fc1_weight, weights[f"{p}.gate_up.weight"])
            put(block.layer.fc2_weight, weights[f"{p}.down.weight"])
