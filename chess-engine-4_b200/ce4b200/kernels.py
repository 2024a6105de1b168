"""Kernel-op API: the operators of ``chess_engine_4.kernels`` on the sm_100a library.

Each function validates its arguments the way the reference does (``ValueError`` for
device, dtype, rank and shape problems; src/chess_engine_4/kernels/dense.py:33-43,
132-139, 366-382) and then calls the C ABI on the tensors' current CUDA stream.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import NamedTuple

import torch

from . import _lib


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _check_bf16_matrix(name: str, tensor: torch.Tensor) -> None:
    if tensor.device.type != "cuda":
        raise ValueError(f"{name} must be a CUDA tensor")
    if tensor.dtype != torch.bfloat16:
        raise ValueError(f"{name} must have dtype torch.bfloat16")
    if tensor.ndim != 2 or not tensor.is_contiguous():
        raise ValueError(f"{name} must be a contiguous matrix")


def _check_bf16_vector(name: str, tensor: torch.Tensor, size: int) -> None:
    if tensor.device.type != "cuda" or tensor.dtype != torch.bfloat16:
        raise ValueError(f"{name} must be a BF16 CUDA tensor")
    if tuple(tensor.shape) != (size,) or not tensor.is_contiguous():
        raise ValueError(f"{name} must be BF16 with shape [{size}]")


def bf16_gemm(left: torch.Tensor, right: torch.Tensor) -> torch.Tensor:
    """``left @ right.T`` in BF16 with FP32 accumulation (tcgen05 GEMM).

    Mirrors ``_bf16_gemm`` (src/chess_engine_4/kernels/dense.py:116-129).
    """

    _check_bf16_matrix("left", left)
    _check_bf16_matrix("right", right)
    if left.shape[1] != right.shape[1]:
        raise ValueError("BF16 GEMM reduction dimensions do not match")
    if right.shape[0] % 16:
        raise ValueError("BF16 GEMM output columns must be a multiple of 16")
    if left.shape[1] % 8:
        raise ValueError("BF16 GEMM reduction dimension must be a multiple of 8")
    out = torch.empty(left.shape[0], right.shape[0], dtype=torch.bfloat16, device=left.device)
    lib = _lib.library()
    with torch.cuda.device(left.device):
        _lib.check(
            lib.ce4b_bf16_gemm(
                left.data_ptr(),
                right.data_ptr(),
                out.data_ptr(),
                left.shape[0],
                right.shape[0],
                left.shape[1],
                _stream(left),
            )
        )
    return out


def rmsnorm_forward(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """Row RMSNorm, BF16 in/out, FP32 math (kernels/src/sm100/dense.cu:313-348)."""

    _check_bf16_matrix("x", x)
    _check_bf16_vector("weight", weight, x.shape[1])
    out = torch.empty_like(x)
    with torch.cuda.device(x.device):
        _lib.check(
            _lib.library().ce4b_rmsnorm_forward(
                x.data_ptr(), weight.data_ptr(), out.data_ptr(), x.shape[0], x.shape[1], eps,
                _stream(x),
            )
        )
    return out


def swiglu_forward(gate_up: torch.Tensor) -> torch.Tensor:
    """``silu(gate) * up`` over a ``[rows, 2H]`` gate|up tensor (sm100/dense.cu:350-377)."""

    _check_bf16_matrix("gate_up", gate_up)
    if gate_up.shape[1] % 2:
        raise ValueError("gate_up must have an even number of columns")
    hidden_dim = gate_up.shape[1] // 2
    hidden = torch.empty(gate_up.shape[0], hidden_dim, dtype=torch.bfloat16, device=gate_up.device)
    with torch.cuda.device(gate_up.device):
        _lib.check(
            _lib.library().ce4b_swiglu_forward(
                gate_up.data_ptr(), hidden.data_ptr(), gate_up.shape[0], hidden_dim,
                _stream(gate_up),
            )
        )
    return hidden


def residual_add(out: torch.Tensor, residual: torch.Tensor) -> torch.Tensor:
    """In place ``out = bf16(out + residual)`` (sm100/dense.cu:379-390)."""

    _check_bf16_matrix("out", out)
    _check_bf16_matrix("residual", residual)
    if out.shape != residual.shape:
        raise ValueError("residual must match out")
    with torch.cuda.device(out.device):
        _lib.check(
            _lib.library().ce4b_residual_add(
                out.data_ptr(), residual.data_ptr(), out.numel(), _stream(out)
            )
        )
    return out


def dense_block_forward(
    x: torch.Tensor,
    norm_weight: torch.Tensor,
    gate_up_weight: torch.Tensor,
    down_weight: torch.Tensor,
    *,
    precision: str,
    eps: float = 1e-6,
) -> torch.Tensor:
    """One dense SwiGLU residual block: ``x + down(swiglu(gate_up(rmsnorm(x))))``.

    Same arguments and checks as the reference operator
    (src/chess_engine_4/kernels/dense.py:141-160, 357-392), except that any expansion
    ratio whose hidden width is a multiple of 64 (128 for MXFP8) is accepted (the
    reference custom path requires ratio 4).

    ``precision="mxfp8"`` follows the reference's recipe step by step (dense.py:395-407):
    the RMSNorm output and both weights are quantised per call (``quantize_mxfp8``), the
    gate_up product is a block-scaled GEMM with a BF16 output, SwiGLU runs in BF16, the
    hidden activations and the down weight are quantised and multiplied the same way, and
    the residual is added last; every step is one of this library's kernels.
    """

    _check_bf16_matrix("x", x)
    d_model = x.shape[1]
    if precision not in ("bf16", "mxfp8"):
        raise ValueError(f"custom dense kernel does not support precision={precision!r}")
    _check_bf16_vector("norm_weight", norm_weight, d_model)
    _check_bf16_matrix("gate_up_weight", gate_up_weight)
    _check_bf16_matrix("down_weight", down_weight)
    hidden_dim = down_weight.shape[1]
    if tuple(gate_up_weight.shape) != (2 * hidden_dim, d_model):
        raise ValueError(f"gate_up_weight must have shape [{2 * hidden_dim}, {d_model}]")
    if tuple(down_weight.shape) != (d_model, hidden_dim):
        raise ValueError(f"down_weight must have shape [{d_model}, {hidden_dim}]")
    if precision == "mxfp8":
        for name, t in (("x", x), ("gate_up_weight", gate_up_weight), ("down_weight", down_weight)):
            if any(size % MXFP8_TILE_SIZE for size in t.shape):
                raise ValueError(f"{name} dimensions must be multiples of {MXFP8_TILE_SIZE}")
        normalized = rmsnorm_forward(x, norm_weight, eps)
        gate_up = mxfp8_gemm(quantize_mxfp8(normalized), quantize_mxfp8(gate_up_weight))
        hidden = swiglu_forward(gate_up)
        projected = mxfp8_gemm(quantize_mxfp8(hidden), quantize_mxfp8(down_weight))
        return residual_add(projected, x)
    lib = _lib.library()
    rows = x.shape[0]
    ws_bytes = lib.ce4b_dense_block_workspace_size(rows, d_model, hidden_dim)
    if ws_bytes < 0:
        raise ValueError("invalid dense block extents")
    workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device)
    out = torch.empty_like(x)
    with torch.cuda.device(x.device):
        _lib.check(
            lib.ce4b_dense_block_forward(
                x.data_ptr(),
                norm_weight.data_ptr(),
                gate_up_weight.data_ptr(),
                down_weight.data_ptr(),
                out.data_ptr(),
                workspace.data_ptr(),
                rows,
                d_model,
                hidden_dim,
                eps,
                _lib.PRECISION_BF16,
                _stream(x),
            )
        )
    return out


MXFP8_TILE_SIZE = 128


@dataclass(frozen=True, slots=True)
class Mxfp8Tensor:
    """E4M3 codes and their E8M0 scale tiles (src/chess_engine_4/kernels/dense.py:27-30)."""

    values: torch.Tensor  # float8_e4m3fn [rows, cols]
    scales: torch.Tensor  # uint8 [rows/128, cols/128, 32, 16]


def _check_mx_matrix(name: str, tensor: torch.Tensor) -> None:
    _check_bf16_matrix(name, tensor)
    if any(size % MXFP8_TILE_SIZE for size in tensor.shape):
        raise ValueError(f"{name} dimensions must be multiples of {MXFP8_TILE_SIZE}")


def quantize_mxfp8(tensor: torch.Tensor) -> Mxfp8Tensor:
    """MXFP8 quantisation, bit-exact to the reference recipe (kernels/dense.py:46-60)."""

    _check_mx_matrix("tensor", tensor)
    rows, cols = tensor.shape
    values = torch.empty_like(tensor, dtype=torch.float8_e4m3fn)
    scales = torch.empty(rows // 128, cols // 128, 32, 16, dtype=torch.uint8, device=tensor.device)
    with torch.cuda.device(tensor.device):
        _lib.check(
            _lib.library().ce4b_quantize_mxfp8(
                tensor.data_ptr(), values.data_ptr(), scales.data_ptr(), rows, cols, _stream(tensor)
            )
        )
    return Mxfp8Tensor(values=values, scales=scales)


def quantize_mxfp8_transpose(tensor: torch.Tensor) -> Mxfp8Tensor:
    """MXFP8 quantisation of ``tensor.T`` without materialising the BF16 transpose
    (kernels/dense.py:63-84): values [cols, rows], scales [cols/128, rows/128, 32, 16]."""

    _check_mx_matrix("tensor", tensor)
    rows, cols = tensor.shape
    values = torch.empty(cols, rows, dtype=torch.float8_e4m3fn, device=tensor.device)
    scales = torch.empty(cols // 128, rows // 128, 32, 16, dtype=torch.uint8, device=tensor.device)
    with torch.cuda.device(tensor.device):
        _lib.check(
            _lib.library().ce4b_quantize_mxfp8_transpose(
                tensor.data_ptr(), values.data_ptr(), scales.data_ptr(), rows, cols, _stream(tensor)
            )
        )
    return Mxfp8Tensor(values=values, scales=scales)


def mxfp8_gemm(left: Mxfp8Tensor, right: Mxfp8Tensor) -> torch.Tensor:
    """``dequant(left) @ dequant(right).T`` in BF16 on block-scaled tcgen05 MMAs
    (replaces kernels/dense.py:87-113; any output width divisible by 128)."""

    rows, reduction = left.values.shape
    out_cols, right_reduction = right.values.shape
    if reduction != right_reduction:
        raise ValueError("MXFP8 GEMM reduction dimensions do not match")
    for t in (left.values, right.values):
        if t.device.type != "cuda" or t.dtype != torch.float8_e4m3fn or not t.is_contiguous():
            raise ValueError("MXFP8 values must be contiguous float8_e4m3fn CUDA tensors")
    if rows % 128 or out_cols % 128 or reduction % 128:
        raise ValueError("MXFP8 GEMM dimensions must be multiples of 128")
    out = torch.empty(rows, out_cols, dtype=torch.bfloat16, device=left.values.device)
    with torch.cuda.device(out.device):
        _lib.check(
            _lib.library().ce4b_mxfp8_gemm(
                left.values.data_ptr(), left.scales.data_ptr(), right.values.data_ptr(),
                right.scales.data_ptr(), out.data_ptr(), rows, out_cols, reduction, _stream(out),
            )
        )
    return out


EXPERT_COUNT = 64
MOE_ROW_ALIGNMENT = 128


def moe_forward(
    x: torch.Tensor,
    gate_up_weight: torch.Tensor,
    down_weight: torch.Tensor,
    route_probs: torch.Tensor,
    expert_offsets: torch.Tensor,
) -> torch.Tensor:
    """Expert SwiGLU MLP over rows sorted and padded by expert.

    Mirrors ``moe_forward`` (src/chess_engine_4/kernels/moe.py:24-46): rows
    ``expert_offsets[e]:expert_offsets[e+1]`` of ``x`` go through expert ``e`` and are
    scaled by ``route_probs``. Segments must start on multiples of 128 rows (the reference's
    static dispatch pads to 128, src/chess_engine_4/model/moe.py:239-251); rows past
    ``expert_offsets[64]`` are left unwritten.
    """

    _check_bf16_matrix("x", x)
    rows, d_model = x.shape
    if gate_up_weight.ndim != 3 or gate_up_weight.shape[0] != EXPERT_COUNT:
        raise ValueError("gate_up_weight must be [64, 2H, d]")
    hidden_dim = gate_up_weight.shape[1] // 2
    if tuple(gate_up_weight.shape) != (EXPERT_COUNT, 2 * hidden_dim, d_model):
        raise ValueError(f"gate_up_weight must have shape [64, {2 * hidden_dim}, {d_model}]")
    if tuple(down_weight.shape) != (EXPERT_COUNT, d_model, hidden_dim):
        raise ValueError(f"down_weight must have shape [64, {d_model}, {hidden_dim}]")
    for name, t in (("gate_up_weight", gate_up_weight), ("down_weight", down_weight)):
        if t.dtype != torch.bfloat16 or not t.is_contiguous() or t.device != x.device:
            raise ValueError(f"{name} must be a contiguous BF16 tensor on x's device")
    if route_probs.dtype != torch.bfloat16 or tuple(route_probs.shape) != (rows,):
        raise ValueError("route_probs must be BF16 with one entry per row")
    if expert_offsets.dtype != torch.int32 or tuple(expert_offsets.shape) != (EXPERT_COUNT + 1,):
        raise ValueError("expert_offsets must be int32 [65]")
    lib = _lib.library()
    ws = torch.empty(lib.ce4b_moe_workspace_size(rows, d_model, hidden_dim), dtype=torch.uint8, device=x.device)
    out = torch.empty_like(x)
    with torch.cuda.device(x.device):
        _lib.check(
            lib.ce4b_moe_forward(
                x.data_ptr(), gate_up_weight.data_ptr(), down_weight.data_ptr(),
                route_probs.contiguous().data_ptr(), expert_offsets.contiguous().data_ptr(),
                out.data_ptr(), ws.data_ptr(), rows, d_model, hidden_dim, _stream(x),
            )
        )
    return out


def moe_route(
    logits: torch.Tensor, qb_beta: torch.Tensor
) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Quantile-balanced top-2 selection of the reference's eval path
    (src/chess_engine_4/model/moe.py:50-63, 160-177): experts = top-2 of (logits - beta)
    with the lower index winning ties, weights = softmax(logits)[experts] rounded to BF16.

    Returns (experts int32 [T, 2], weights float32 [T, 2], tokens_per_expert int32 [64]).
    """

    if logits.device.type != "cuda" or logits.dtype != torch.bfloat16:
        raise ValueError("logits must be a BF16 CUDA tensor")
    if logits.ndim != 2 or logits.shape[1] != EXPERT_COUNT or not logits.is_contiguous():
        raise ValueError("logits must be a contiguous [T, 64] matrix")
    beta = qb_beta.to(device=logits.device, dtype=torch.float32).contiguous()
    if tuple(beta.shape) != (EXPERT_COUNT,):
        raise ValueError("qb_beta must have 64 entries")
    tokens = logits.shape[0]
    experts = torch.empty(tokens, 2, dtype=torch.int32, device=logits.device)
    probs = torch.empty(tokens, 2, dtype=torch.float32, device=logits.device)
    counts = torch.zeros(EXPERT_COUNT, dtype=torch.int32, device=logits.device)
    with torch.cuda.device(logits.device):
        _lib.check(
            _lib.library().ce4b_moe_route(
                logits.data_ptr(), beta.data_ptr(), experts.data_ptr(), probs.data_ptr(),
                counts.data_ptr(), tokens, _stream(logits),
            )
        )
    return experts, probs, counts


class MoeDispatch(NamedTuple):
    """Result of :func:`moe_route_dispatch` (all on the input's device)."""

    logits: torch.Tensor          # BF16 [T, 64]: the router logits the selection used
    experts: torch.Tensor         # int32 [T, 2]: best expert first
    probs: torch.Tensor           # float32 [T, 2]: BF16-rounded routing weights
    positions: torch.Tensor       # int32 [T, 2]: row of each route in the permuted layout
    expert_offsets: torch.Tensor  # int32 [65]: segment starts (multiples of 128), then the total
    counts: torch.Tensor          # int32 [64]: routes per expert
    rows: torch.Tensor            # BF16 [capacity, d]: permuted rows (padding rows unwritten)
    row_probs: torch.Tensor       # float32 [capacity]: routing weight of each permuted row


def moe_route_dispatch(n: torch.Tensor, router_weight: torch.Tensor, qb_beta: torch.Tensor) -> MoeDispatch:
    """Routing and static dispatch of one MoE layer with the forward's own kernels (router
    GEMM + top-2 epilogue, histogram scan, dispatch): ``MoeBlock.forward``'s eval-path
    selection and ``_run_experts_static`` placement (src/chess_engine_4/model/moe.py:36-47,
    160-177, 232-267). Routes are ordered by ``2 * token + k`` within each expert, and
    every expert segment starts on a multiple of 128 rows."""

    _check_bf16_matrix("n", n)
    tokens, d_model = n.shape
    if tuple(router_weight.shape) != (EXPERT_COUNT, d_model) or router_weight.dtype != torch.bfloat16:
        raise ValueError(f"router_weight must be BF16 [64, {d_model}]")
    if not router_weight.is_contiguous() or router_weight.device != n.device:
        raise ValueError("router_weight must be contiguous and on n's device")
    beta = qb_beta.to(device=n.device, dtype=torch.float32).contiguous()
    if tuple(beta.shape) != (EXPERT_COUNT,):
        raise ValueError("qb_beta must have 64 entries")
    lib = _lib.library()
    cap = lib.ce4b_moe_dispatch_capacity(tokens)
    dev = n.device
    out = MoeDispatch(
        logits=torch.empty(tokens, EXPERT_COUNT, dtype=torch.bfloat16, device=dev),
        experts=torch.empty(tokens, 2, dtype=torch.int32, device=dev),
        probs=torch.empty(tokens, 2, dtype=torch.float32, device=dev),
        positions=torch.empty(tokens, 2, dtype=torch.int32, device=dev),
        expert_offsets=torch.empty(EXPERT_COUNT + 1, dtype=torch.int32, device=dev),
        counts=torch.empty(EXPERT_COUNT, dtype=torch.int32, device=dev),
        rows=torch.empty(cap, d_model, dtype=torch.bfloat16, device=dev),
        row_probs=torch.empty(cap, dtype=torch.float32, device=dev),
    )
    ws = torch.empty(lib.ce4b_moe_route_dispatch_workspace_size(tokens), dtype=torch.uint8, device=dev)
    with torch.cuda.device(dev):
        _lib.check(
            lib.ce4b_moe_route_dispatch(
                n.data_ptr(), router_weight.data_ptr(), beta.data_ptr(), out.logits.data_ptr(),
                out.experts.data_ptr(), out.probs.data_ptr(), out.positions.data_ptr(),
                out.expert_offsets.data_ptr(), out.counts.data_ptr(), out.rows.data_ptr(),
                out.row_probs.data_ptr(), ws.data_ptr(), tokens, d_model, _stream(n),
            )
        )
    return out


def policy_softmax(
    policy: torch.Tensor, move_offsets: torch.Tensor, move_indices: torch.Tensor, temperature: float = 1.0
) -> torch.Tensor:
    """Legal-move probabilities on the device: for position b, softmax((logit - max) *
    temperature) over policy[b, move_indices[move_offsets[b]:move_offsets[b + 1]]]
    (third_party/lc0/src/neural/backends/ce4/backend.cc:182-195)."""

    if policy.dim() != 2 or policy.dtype != torch.float32 or not policy.is_cuda:
        raise ValueError("policy must be a CUDA float32 [B, P] tensor")
    batch, size = policy.shape
    offsets = move_offsets.to(device=policy.device, dtype=torch.int32).contiguous()
    indices = move_indices.to(device=policy.device, dtype=torch.int32).contiguous()
    if offsets.shape != (batch + 1,):
        raise ValueError("move_offsets must have B + 1 entries")
    probs = torch.empty(indices.numel(), dtype=torch.float32, device=policy.device)
    stream = torch.cuda.current_stream(policy.device).cuda_stream
    _lib.check(_lib.library().ce4b_policy_softmax(
        policy.contiguous().data_ptr(), batch, size, offsets.data_ptr(), indices.data_ptr(),
        float(temperature), probs.data_ptr(), stream))
    return probs
