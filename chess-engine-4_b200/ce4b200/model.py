"""Drop-in model API: ``DenseChessNet`` / ``Moe64A2ChessNet`` on the sm_100a library.

The classes keep the reference's configuration dataclasses, constructor arguments,
parameter names (the Transformer Engine module names that checkpoints and
``release/export.py`` use) and ``forward(planes) -> ChessNetOutput`` contract:

* src/chess_engine_4/model/dense.py:34-82, 85-203  (dense tower)
* src/chess_engine_4/model/moe.py:74-106, 109-180, 337-415  (moe64a2 tower)
* src/chess_engine_4/model/output.py:10-16, registry.py:25-77

``forward`` runs entirely in libce4b200 (tcgen05 GEMMs with fused epilogues); the
PyTorch parameters are the source of truth and are uploaded into the library's weight
arena whenever they change. Inference only: no autograd graph is recorded.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, fields
from typing import Any, ClassVar, Literal, cast

import torch
from torch import nn

from . import _lib

POLICY_SIZE = 1858
INPUT_PLANE_COUNT = 112
HISTORY_PLANE_COUNT = 104
RULE50_PLANE_INDEX = HISTORY_PLANE_COUNT + 5
BOARD_SIZE = 8
HISTORY_LENGTH = 8
PLANES_PER_HISTORY_POSITION = HISTORY_PLANE_COUNT // HISTORY_LENGTH
SUPPORTED_ACTIVATIONS = frozenset({"geglu", "gelu", "silu", "srelu", "swiglu"})
GATED_ACTIVATIONS = frozenset({"geglu", "swiglu"})
EXPERT_COUNT = 64
ACTIVE_EXPERT_COUNT = 2
DENSE_EXPANSION_RATIO = 4
MXFP8_FEATURE_ALIGNMENT = 32
FUSED_DISPATCH_MIN_WIDTH = 1024

Precision = Literal["bf16", "mxfp8"]
KernelBackend = Literal["custom", "te"]
InputPipeline = Literal["overlap", "pageable", "pinned"]


def mxfp8_aligned_size(size: int) -> int:
    return (size + 31) // 32 * 32


ROUTER_OUTPUT_SIZE = mxfp8_aligned_size(EXPERT_COUNT)


def normalize_lc0_planes(
    planes: torch.Tensor, *, rule50_plane_index: int = RULE50_PLANE_INDEX
) -> torch.Tensor:
    """In-place rule-50 ply / 99 (src/chess_engine_4/model/dense.py:34-42)."""

    planes[:, rule50_plane_index].div_(99.0)
    return planes


def select_lc0_history(planes: torch.Tensor, history_length: int) -> torch.Tensor:
    """Keep recent history and all aux planes (src/chess_engine_4/model/dense.py:45-51)."""

    history_planes = history_length * PLANES_PER_HISTORY_POSITION
    if history_planes == HISTORY_PLANE_COUNT:
        return planes
    return torch.cat((planes[:, :history_planes], planes[:, HISTORY_PLANE_COUNT:]), dim=1)


def model_input_plane_count(history_length: int) -> int:
    auxiliary_planes = INPUT_PLANE_COUNT - HISTORY_PLANE_COUNT
    return history_length * PLANES_PER_HISTORY_POSITION + auxiliary_planes


@dataclass(frozen=True, slots=True)
class ChessNetOutput:
    policy_logits: torch.Tensor
    wdl_logits: torch.Tensor
    moves_left: torch.Tensor
    router_dead_experts: torch.Tensor | None = None
    router_tokens_per_expert: torch.Tensor | None = None


@dataclass(frozen=True, slots=True)
class DenseChessNetConfig:
    """Same fields, defaults and checks as src/chess_engine_4/model/dense.py:59-82."""

    kind: str = "dense"
    history_length: int = HISTORY_LENGTH
    d_model: int = 1024
    depth: int = 8
    expansion_ratio: float = 4.0
    activation: str = "swiglu"
    rms_norm_eps: float = 1e-6
    precision: Precision = "mxfp8"
    kernel_backend: KernelBackend = "te"
    input_pipeline: InputPipeline = "pinned"

    def __post_init__(self) -> None:
        if self.d_model < 64:
            raise ValueError("d_model must be at least 64")
        if not 1 <= self.history_length <= HISTORY_LENGTH:
            raise ValueError(f"history_length must be in [1, {HISTORY_LENGTH}]")
        if self.expansion_ratio <= 0:
            raise ValueError("expansion_ratio must be positive")
        if self.activation not in SUPPORTED_ACTIVATIONS:
            choices = ", ".join(sorted(SUPPORTED_ACTIVATIONS))
            raise ValueError(f"unsupported activation {self.activation!r}; choose from {choices}")


@dataclass(frozen=True, slots=True)
class Moe64A2ChessNetConfig:
    """Same fields, defaults and checks as src/chess_engine_4/model/moe.py:74-106."""

    kind: str = "moe64a2"
    history_length: int = HISTORY_LENGTH
    d_model: int = 1024
    depth: int = 8
    expansion_ratio: float = 2.0
    activation: str = "swiglu"
    rms_norm_eps: float = 1e-6
    precision: Precision = "mxfp8"
    kernel_backend: KernelBackend = "te"
    input_pipeline: InputPipeline = "pinned"

    num_experts: ClassVar[int] = EXPERT_COUNT
    num_active_experts: ClassVar[int] = ACTIVE_EXPERT_COUNT

    def __post_init__(self) -> None:
        if self.d_model < 64:
            raise ValueError("d_model must be at least 64")
        if not 1 <= self.history_length <= HISTORY_LENGTH:
            raise ValueError(f"history_length must be in [1, {HISTORY_LENGTH}]")
        if self.d_model % MXFP8_FEATURE_ALIGNMENT != 0:
            raise ValueError(f"d_model must be divisible by {MXFP8_FEATURE_ALIGNMENT}")
        if self.expansion_ratio <= 0:
            raise ValueError("expansion_ratio must be positive")
        if self.depth <= 0 or self.depth % 2 != 0:
            raise ValueError("moe64a2 depth must be a positive even number")
        if self.activation != "swiglu":
            raise ValueError("moe64a2 only supports activation='swiglu'")

    @property
    def cuda_graph_compatible(self) -> bool:
        return self.d_model < FUSED_DISPATCH_MIN_WIDTH


type ModelConfig = DenseChessNetConfig | Moe64A2ChessNetConfig

_FIXED_LC0_GEOMETRY = {
    "input_planes": INPUT_PLANE_COUNT,
    "board_size": BOARD_SIZE,
    "policy_size": POLICY_SIZE,
}


def model_config_from_dict(values: dict[str, Any]) -> ModelConfig:
    """Parse a ``[model]`` mapping (src/chess_engine_4/model/registry.py:25-36, 66-77)."""

    values = dict(values)
    for name, expected in _FIXED_LC0_GEOMETRY.items():
        actual = values.pop(name, expected)
        if actual != expected:
            raise ValueError(f"[model].{name} must be {expected}, got {actual!r}.")
    kind = values.get("kind", "dense")
    section: type[Any]
    if kind == "dense":
        section = DenseChessNetConfig
    elif kind == "moe64a2":
        section = Moe64A2ChessNetConfig
    else:
        raise ValueError(f"unknown model kind: {kind}")
    names = {f.name for f in fields(section)}
    unknown = sorted(set(values) - names)
    if unknown:
        raise ValueError(f"[model] has unknown key(s): {', '.join(unknown)}.")
    return cast(ModelConfig, section(**values))


def dense_parameter_count(
    *,
    history_length: int = HISTORY_LENGTH,
    d_model: int,
    depth: int,
    expansion_ratio: float = 4.0,
    activation: str = "geglu",
) -> int:
    """Parameter count of the dense tower (src/chess_engine_4/model/dense.py:206-226)."""

    input_dim = model_input_plane_count(history_length) * BOARD_SIZE**2
    hidden_dim = int(d_model * expansion_ratio)
    projection_count = 3 if activation in GATED_ACTIVATIONS else 2
    block_params = depth * (projection_count * d_model * hidden_dim)
    norm_params = (depth + 1) * d_model
    input_params = input_dim * d_model + d_model
    aligned_policy_size = mxfp8_aligned_size(POLICY_SIZE)
    head_params = d_model * aligned_policy_size + aligned_policy_size + 2 * (d_model * 32 + 32)
    return input_params + block_params + norm_params + head_params


def moe64a2_parameter_count(
    *,
    history_length: int = HISTORY_LENGTH,
    d_model: int,
    depth: int,
    expansion_ratio: float = 2.0,
) -> int:
    """Parameter count of the moe64a2 tower (src/chess_engine_4/model/moe.py:418-449)."""

    if depth <= 0 or depth % 2 != 0:
        raise ValueError("moe64a2 depth must be a positive even number")
    input_dim = model_input_plane_count(history_length) * BOARD_SIZE**2
    hidden_dim = int(d_model * expansion_ratio)
    half = depth // 2
    expert_params = half * EXPERT_COUNT * 3 * d_model * hidden_dim
    router_params = half * d_model * ROUTER_OUTPUT_SIZE
    dense_params = half * 3 * d_model * (DENSE_EXPANSION_RATIO * d_model)
    norm_params = (depth + 1) * d_model
    aligned_policy_size = mxfp8_aligned_size(POLICY_SIZE)
    head_params = d_model * aligned_policy_size + aligned_policy_size + 2 * (d_model * 32 + 32)
    return (
        input_dim * d_model
        + d_model
        + expert_params
        + router_params
        + dense_params
        + norm_params
        + head_params
    )


# ---------------------------------------------------------------- parameter containers
# These modules only hold parameters under the reference's (Transformer Engine) names;
# all computation happens in libce4b200.


def _normal_(t: torch.Tensor, std: float = 0.02) -> torch.Tensor:
    with torch.no_grad():
        return t.normal_(0.0, std)


class Linear(nn.Module):
    """Holds ``weight [out, in]`` and optional ``bias [out]`` (te.Linear names)."""

    def __init__(self, in_features: int, out_features: int, *, bias: bool = True) -> None:
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.weight = nn.Parameter(_normal_(torch.empty(out_features, in_features, dtype=torch.bfloat16)))
        self.bias = (
            nn.Parameter(torch.zeros(out_features, dtype=torch.bfloat16)) if bias else None
        )


class RMSNorm(nn.Module):
    """Holds ``weight [d]`` (te.RMSNorm names)."""

    def __init__(self, d_model: int, eps: float) -> None:
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(d_model, dtype=torch.bfloat16))


class LayerNormMLP(nn.Module):
    """Holds ``layer_norm_weight [d]``, ``fc1_weight [2h, d]``, ``fc2_weight [d, h]``
    (te.LayerNormMLP names; fc1 rows 0..h-1 are the SwiGLU gate, h..2h-1 the up)."""

    def __init__(self, d_model: int, hidden_dim: int) -> None:
        super().__init__()
        self.layer_norm_weight = nn.Parameter(torch.ones(d_model, dtype=torch.bfloat16))
        self.fc1_weight = nn.Parameter(
            _normal_(torch.empty(2 * hidden_dim, d_model, dtype=torch.bfloat16))
        )
        self.fc2_weight = nn.Parameter(
            _normal_(torch.empty(d_model, hidden_dim, dtype=torch.bfloat16))
        )


class DenseBlock(nn.Module):
    """Dense SwiGLU residual block (src/chess_engine_4/model/dense.py:85-135)."""

    def __init__(
        self,
        d_model: int,
        hidden_dim: int,
        rms_norm_eps: float,
        activation: str,
        precision: Precision,
    ) -> None:
        super().__init__()
        if activation != "swiglu":
            raise ValueError("the sm_100a forward supports activation='swiglu' only")
        self.d_model = d_model
        self.hidden_dim = hidden_dim
        self.rms_norm_eps = rms_norm_eps
        self.activation = activation
        self.precision = precision
        self.layer = LayerNormMLP(d_model, hidden_dim)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        from .kernels import dense_block_forward

        return dense_block_forward(
            x,
            self.layer.layer_norm_weight,
            self.layer.fc1_weight,
            self.layer.fc2_weight,
            precision=self.precision,
            eps=self.rms_norm_eps,
        )

    def enable_custom_kernels(self) -> None:
        """The block always runs on the sm_100a kernels; kept for API compatibility."""


class GroupedLinear(nn.Module):
    """Holds ``weight0 .. weight{E-1}`` of shape ``[out, in]`` (te.ops.GroupedLinear names)."""

    def __init__(self, num_groups: int, in_features: int, out_features: int) -> None:
        super().__init__()
        self.num_groups = num_groups
        for e in range(num_groups):
            self.register_parameter(
                f"weight{e}",
                nn.Parameter(_normal_(torch.empty(out_features, in_features, dtype=torch.bfloat16))),
            )

    def stacked(self) -> torch.Tensor:
        return torch.stack([getattr(self, f"weight{e}") for e in range(self.num_groups)])


class ScaledSwiGLU(nn.Module):
    """Parameter-free placeholder at index 1 of the expert sequence (te.ops.ScaledSwiGLU)."""


class MoeBlock(nn.Module):
    """Top-2 64-expert block with quantile-balanced routing (src/chess_engine_4/model/moe.py:109-180)."""

    def __init__(self, config: Moe64A2ChessNetConfig) -> None:
        super().__init__()
        hidden_dim = int(config.d_model * config.expansion_ratio)
        if hidden_dim % MXFP8_FEATURE_ALIGNMENT != 0:
            raise ValueError(
                f"expert hidden dimension must be divisible by {MXFP8_FEATURE_ALIGNMENT}"
            )
        self.d_model = config.d_model
        self.hidden_dim = hidden_dim
        self.norm = RMSNorm(config.d_model, config.rms_norm_eps)
        self.router = Linear(config.d_model, ROUTER_OUTPUT_SIZE, bias=False)
        self.router_qb_beta: torch.Tensor
        self.register_buffer("router_qb_beta", torch.zeros(EXPERT_COUNT, dtype=torch.float32))
        self.experts = nn.Sequential(
            GroupedLinear(EXPERT_COUNT, config.d_model, 2 * hidden_dim),
            ScaledSwiGLU(),
            GroupedLinear(EXPERT_COUNT, hidden_dim, config.d_model),
        )

    def enable_custom_kernels(self) -> None:
        """The block always runs on the sm_100a kernels; kept for API compatibility."""


# ---------------------------------------------------------------- native engine handle
class _NativeModel:
    """Owns one ``ce4b_model`` handle (weights + workspace on one GPU)."""

    def __init__(self, cfg: _lib.ModelConfigStruct, device: int, max_batch: int) -> None:
        self.lib = _lib.library()
        self.device = device
        self.max_batch = max_batch
        handle = ctypes.c_void_p()
        _lib.check(self.lib.ce4b_model_create(ctypes.byref(cfg), device, max_batch, ctypes.byref(handle)))
        self.handle = handle

    def set_latency_path(self, enabled: bool) -> None:
        _lib.check(self.lib.ce4b_model_set_latency_path(self.handle, 1 if enabled else 0))

    def uses_latency_path(self, batch: int) -> bool:
        uses = ctypes.c_int32()
        _lib.check(self.lib.ce4b_model_uses_latency_path(self.handle, batch, ctypes.byref(uses)))
        return bool(uses.value)

    def upload(self, tensors: dict[str, torch.Tensor]) -> None:
        target = torch.device("cuda", self.device)
        staged: dict[str, torch.Tensor] = {}
        for name, tensor in tensors.items():
            if tensor.dtype not in (torch.float32, torch.bfloat16):
                raise ValueError(f"tensor {name} must be BF16 or FP32, got {tensor.dtype}")
            t = tensor.detach()
            if t.device.type == "cuda":
                t = t.to(device=target)
            staged[name] = t.contiguous()
        # The library copies with the synchronous cudaMemcpy, outside PyTorch's streams.
        torch.cuda.synchronize(target)
        for name, t in staged.items():
            dtype = _lib.DTYPE_F32 if t.dtype == torch.float32 else _lib.DTYPE_BF16
            shape = (ctypes.c_int64 * t.ndim)(*t.shape)
            src_is_device = 1 if t.device.type == "cuda" else 0
            _lib.check(
                self.lib.ce4b_model_set_tensor(
                    self.handle, name.encode(), t.data_ptr(), dtype, t.ndim, shape, src_is_device
                )
            )
        _lib.check(self.lib.ce4b_model_finalize(self.handle))

    def forward(
        self,
        layout: int,
        data: torch.Tensor,
        scalars: torch.Tensor | None,
        batch: int,
        *,
        wdl_probs: bool,
        normalize_in_place: bool,
        tokens_per_expert: torch.Tensor | None = None,
    ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        dev = torch.device("cuda", self.device)
        policy = torch.empty(batch, POLICY_SIZE, dtype=torch.float32, device=dev)
        wdl = torch.empty(batch, 3, dtype=torch.float32, device=dev)
        moves_left = torch.empty(batch, dtype=torch.float32, device=dev)
        stream = torch.cuda.current_stream(dev).cuda_stream
        _lib.check(
            self.lib.ce4b_model_forward(
                self.handle,
                layout,
                data.data_ptr(),
                scalars.data_ptr() if scalars is not None else None,
                batch,
                policy.data_ptr(),
                wdl.data_ptr(),
                moves_left.data_ptr(),
                1 if wdl_probs else 0,
                1 if normalize_in_place else 0,
                tokens_per_expert.data_ptr() if tokens_per_expert is not None else None,
                stream,
            )
        )
        return policy, wdl, moves_left

    def enable_expert_parallel(self, rank: int, world: int, unique_id: bytes) -> None:
        if len(unique_id) != 128:
            raise ValueError("the NCCL unique id has 128 bytes")
        buf = ctypes.create_string_buffer(unique_id, 128)
        _lib.check(self.lib.ce4b_model_enable_expert_parallel(self.handle, rank, world, buf))

    def __del__(self) -> None:
        handle = getattr(self, "handle", None)
        if handle is not None and handle.value:
            self.lib.ce4b_model_destroy(handle)
            self.handle = None


class _NativeForwardMixin(nn.Module):
    """Shared engine plumbing of the two tower classes."""

    config: ModelConfig
    _arch: int

    def _native_config(self) -> _lib.ModelConfigStruct:
        cfg = self.config
        precision = _lib.PRECISION_BF16 if cfg.precision == "bf16" else _lib.PRECISION_MXFP8
        return _lib.ModelConfigStruct(
            arch=self._arch,
            d_model=cfg.d_model,
            depth=cfg.depth,
            history_length=cfg.history_length,
            expansion_ratio=float(cfg.expansion_ratio),
            rms_norm_eps=float(cfg.rms_norm_eps),
            policy_size=POLICY_SIZE,
            policy_storage_size=mxfp8_aligned_size(POLICY_SIZE),
            precision=precision,
        )

    def _weights_signature(self) -> tuple[Any, ...]:
        return tuple(
            (t.data_ptr(), t._version, t.device.index) for t in self.state_dict(keep_vars=True).values()
        )

    def _engine(self, batch: int, device: torch.device) -> _NativeModel:
        if device.type != "cuda":
            raise ValueError("planes must be a CUDA tensor (the sm_100a forward has no CPU path)")
        engine: _NativeModel | None = self.__dict__.get("_native")
        index = device.index if device.index is not None else torch.cuda.current_device()
        if engine is None or engine.device != index or engine.max_batch < batch:
            if self.__dict__.get("_ep") is not None:
                raise ValueError(
                    f"expert-parallel model: batch {batch} on cuda:{index} exceeds the engine "
                    "given to enable_expert_parallel"
                )
            capacity = max(batch, engine.max_batch if engine is not None else 0)
            capacity = (capacity + 255) // 256 * 256
            self.__dict__["_native"] = None
            engine = _NativeModel(self._native_config(), index, capacity)
            engine.set_latency_path(self.__dict__.get("_latency_path", True))
            self.__dict__["_native"] = engine
            self.__dict__["_native_signature"] = None
        signature = self._weights_signature()
        if self.__dict__.get("_native_signature") != signature:
            engine.upload(self.safetensors_tensors())
            self.__dict__["_native_signature"] = signature
        return engine

    def safetensors_tensors(self) -> dict[str, torch.Tensor]:
        raise NotImplementedError

    def _run(
        self,
        layout: int,
        data: torch.Tensor,
        scalars: torch.Tensor | None,
        *,
        wdl_probs: bool = False,
        normalize_in_place: bool = False,
    ) -> ChessNetOutput:
        batch = data.shape[0]
        if batch == 0:
            raise ValueError("batch must contain at least one position")
        engine = self._engine(batch, data.device)
        tokens = None
        if self._arch == _lib.ARCH_MOE64A2:
            tokens = torch.empty(self.config.depth // 2, EXPERT_COUNT, dtype=torch.int32, device=data.device)
        with torch.no_grad():
            policy, wdl, moves_left = engine.forward(
                layout,
                data,
                scalars,
                batch,
                wdl_probs=wdl_probs,
                normalize_in_place=normalize_in_place,
                tokens_per_expert=tokens,
            )
        if tokens is None:
            return ChessNetOutput(policy_logits=policy, wdl_logits=wdl, moves_left=moves_left)
        tokens64 = tokens.to(torch.int64)
        return ChessNetOutput(
            policy_logits=policy,
            wdl_logits=wdl,
            moves_left=moves_left,
            router_dead_experts=tokens64.eq(0).sum(dim=1).max(),
            router_tokens_per_expert=tokens64,
        )

    def forward(self, planes: torch.Tensor) -> ChessNetOutput:
        """``planes`` float32/bfloat16 ``[B, 112, 8, 8]`` on a CUDA device.

        As in the reference (src/chess_engine_4/model/dense.py:188-192), the rule-50 plane
        of ``planes`` is divided by 99 in place when the full 8-position history is used.
        Outputs are FP32 tensors holding BF16-rounded logits.
        """

        if planes.ndim != 4 or tuple(planes.shape[1:]) != (INPUT_PLANE_COUNT, BOARD_SIZE, BOARD_SIZE):
            raise ValueError("planes must have shape [B, 112, 8, 8]")
        if planes.dtype == torch.float32:
            layout = _lib.INPUT_F32_PLANES
        elif planes.dtype == torch.bfloat16:
            layout = _lib.INPUT_BF16_PLANES
        else:
            raise ValueError(f"planes must be float32 or bfloat16, got {planes.dtype}")
        if planes.is_contiguous():
            return self._run(layout, planes, None, normalize_in_place=True)
        output = self._run(layout, planes.contiguous(), None, normalize_in_place=False)
        if self.config.history_length == HISTORY_LENGTH:
            normalize_lc0_planes(planes)
        return output

    def forward_packed(self, packed_planes: torch.Tensor, plane_scalars: torch.Tensor) -> ChessNetOutput:
        """Training-pipeline input: u8 ``[B, 104, 8]`` bit planes + ``[B, 8]`` scalars
        (src/chess_engine_4/training/packed_input.py:24-47), expanded on the device."""

        if packed_planes.dtype != torch.uint8 or tuple(packed_planes.shape[1:]) != (HISTORY_PLANE_COUNT, BOARD_SIZE):
            raise ValueError("packed_planes must be uint8 [B, 104, 8]")
        if tuple(plane_scalars.shape) != (packed_planes.shape[0], INPUT_PLANE_COUNT - HISTORY_PLANE_COUNT):
            raise ValueError("plane_scalars must be [B, 8]")
        if plane_scalars.dtype == torch.float32:
            layout = _lib.INPUT_PACKED_F32
        elif plane_scalars.dtype == torch.bfloat16:
            layout = _lib.INPUT_PACKED_BF16
        else:
            raise ValueError("plane_scalars must be float32 or bfloat16")
        return self._run(layout, packed_planes.contiguous(), plane_scalars.contiguous())

    def forward_lc0(self, planes: torch.Tensor, *, wdl_probs: bool = True) -> ChessNetOutput:
        """lc0 engine input: ``[B, 112, 2]`` int64 view of ``InputPlane{u64 mask; f32 value}``
        (16 bytes each; see ``ce4b200.synthetic.lc0_planes_tensor``). Returns WDL
        probabilities by default, as Model::Evaluate does (kernels/src/inference/runtime.cu:532-564)."""

        if planes.dtype != torch.int64 or tuple(planes.shape[1:]) != (INPUT_PLANE_COUNT, 2):
            raise ValueError("lc0 planes must be an int64 [B, 112, 2] view of InputPlane records")
        return self._run(_lib.INPUT_LC0, planes.contiguous(), None, wdl_probs=wdl_probs)

    def enable_custom_kernels(self) -> None:
        """Always on the sm_100a kernels; kept for API compatibility."""

    def set_latency_path(self, enabled: bool) -> None:
        """Dense BF16 models with d_model <= 512 run batches of at most 64 positions on the
        small-batch forward (one cooperative launch of transposed tiles spread over the SMs,
        the same folded-RMSNorm arithmetic as the persistent forward). ``False`` sends them to the persistent
        forward instead; the default is ``True``."""

        self.__dict__["_latency_path"] = bool(enabled)
        engine = self.__dict__.get("_native")
        if engine is not None:
            engine.set_latency_path(enabled)


def _bf16(t: torch.Tensor) -> torch.Tensor:
    if t.dtype != torch.bfloat16:
        raise ValueError(f"weights must be BF16, got {t.dtype}")
    return t.detach()


class DenseChessNet(_NativeForwardMixin):
    """Single-token dense model over flattened LCZero input planes
    (src/chess_engine_4/model/dense.py:138-203)."""

    _arch = _lib.ARCH_DENSE

    def __init__(self, config: DenseChessNetConfig | None = None) -> None:
        super().__init__()
        if config is None:
            config = DenseChessNetConfig()
        self.config = config
        input_dim = model_input_plane_count(config.history_length) * BOARD_SIZE**2
        hidden_dim = int(config.d_model * config.expansion_ratio)
        self.input = Linear(input_dim, config.d_model)
        self.blocks = nn.Sequential(
            *[
                DenseBlock(
                    d_model=config.d_model,
                    hidden_dim=hidden_dim,
                    rms_norm_eps=config.rms_norm_eps,
                    activation=config.activation,
                    precision=config.precision,
                )
                for _ in range(config.depth)
            ]
        )
        self.norm = RMSNorm(config.d_model, config.rms_norm_eps)
        self.policy_head = Linear(config.d_model, mxfp8_aligned_size(POLICY_SIZE))
        self.wdl_head = Linear(config.d_model, 32)
        self.moves_left_head = Linear(config.d_model, 32)

    def safetensors_tensors(self) -> dict[str, torch.Tensor]:
        """Weights under the Safetensors v1 names (src/chess_engine_4/release/export.py:164-188)."""

        t: dict[str, torch.Tensor] = _common_tensors(self)
        for i, block in enumerate(self.blocks):
            layer = cast(DenseBlock, block).layer
            t[f"blocks.{i}.norm.weight"] = _bf16(layer.layer_norm_weight)
            t[f"blocks.{i}.gate_up.weight"] = _bf16(layer.fc1_weight)
            t[f"blocks.{i}.down.weight"] = _bf16(layer.fc2_weight)
        return t


class Moe64A2ChessNet(_NativeForwardMixin):
    """Single-token chess model alternating 64-expert and dense layers
    (src/chess_engine_4/model/moe.py:337-415)."""

    _arch = _lib.ARCH_MOE64A2

    def __init__(self, config: Moe64A2ChessNetConfig | None = None) -> None:
        super().__init__()
        if config is None:
            config = Moe64A2ChessNetConfig()
        self.config = config
        self.cuda_graph_compatible = config.cuda_graph_compatible
        input_dim = model_input_plane_count(config.history_length) * BOARD_SIZE**2
        self.input = Linear(input_dim, config.d_model)
        self.blocks = nn.ModuleList(
            [
                MoeBlock(config)
                if layer_index % 2 == 0
                else DenseBlock(
                    d_model=config.d_model,
                    hidden_dim=DENSE_EXPANSION_RATIO * config.d_model,
                    rms_norm_eps=config.rms_norm_eps,
                    activation=config.activation,
                    precision=config.precision,
                )
                for layer_index in range(config.depth)
            ]
        )
        self.norm = RMSNorm(config.d_model, config.rms_norm_eps)
        self.policy_head = Linear(config.d_model, mxfp8_aligned_size(POLICY_SIZE))
        self.wdl_head = Linear(config.d_model, 32)
        self.moves_left_head = Linear(config.d_model, 32)

    def enable_expert_parallel(
        self,
        *,
        max_batch: int,
        device: int | None = None,
        rank: int | None = None,
        world: int | None = None,
        unique_id: bytes | None = None,
    ) -> None:
        """Splits the 64 experts over the ranks (64 / world consecutive experts each, the
        only ones this rank keeps): every MoE layer sends each routed row to its expert's
        rank and the result back over NVLink peer memory, with no host synchronisation.
        Collective: every rank calls it, each with its own GPU. rank / world default to the
        torch.distributed default group, which also carries rank 0's NCCL unique id (used
        once, to exchange the buffer handles) to the others. Later forwards take this
        rank's positions (at most ``max_batch``) and return their outputs, equal to the
        single-GPU forward's; the weights are fixed from then on."""

        if rank is None or world is None:
            import torch.distributed as dist

            rank, world = dist.get_rank(), dist.get_world_size()
        if unique_id is None:
            import torch.distributed as dist

            box = [_lib.nccl_unique_id() if rank == 0 else b""]
            dist.broadcast_object_list(box, src=0)
            unique_id = box[0]
        index = device if device is not None else torch.cuda.current_device()
        self.__dict__["_ep"] = None
        engine = self._engine(max_batch, torch.device("cuda", index))
        engine.enable_expert_parallel(rank, world, unique_id)
        self.__dict__["_ep"] = (rank, world)

    def safetensors_tensors(self) -> dict[str, torch.Tensor]:
        """Weights under the Safetensors v1 names (src/chess_engine_4/release/export.py:96-188)."""

        t: dict[str, torch.Tensor] = _common_tensors(self)
        for i, block in enumerate(self.blocks):
            if isinstance(block, MoeBlock):
                t[f"blocks.{i}.norm.weight"] = _bf16(block.norm.weight)
                t[f"blocks.{i}.router.weight"] = _bf16(block.router.weight)[:EXPERT_COUNT]
                t[f"blocks.{i}.router_qb_beta"] = block.router_qb_beta.detach().float()
                gate_up = cast(GroupedLinear, block.experts[0])
                down = cast(GroupedLinear, block.experts[2])
                t[f"blocks.{i}.experts.gate_up.weight"] = gate_up.stacked().detach()
                t[f"blocks.{i}.experts.down.weight"] = down.stacked().detach()
            else:
                layer = cast(DenseBlock, block).layer
                t[f"blocks.{i}.norm.weight"] = _bf16(layer.layer_norm_weight)
                t[f"blocks.{i}.gate_up.weight"] = _bf16(layer.fc1_weight)
                t[f"blocks.{i}.down.weight"] = _bf16(layer.fc2_weight)
        return t


def _common_tensors(model: DenseChessNet | Moe64A2ChessNet) -> dict[str, torch.Tensor]:
    assert model.input.bias is not None
    assert model.policy_head.bias is not None
    assert model.wdl_head.bias is not None
    assert model.moves_left_head.bias is not None
    return {
        "input.weight": _bf16(model.input.weight),
        "input.bias": _bf16(model.input.bias),
        "final_norm.weight": _bf16(model.norm.weight),
        "policy.weight": _bf16(model.policy_head.weight),
        "policy.bias": _bf16(model.policy_head.bias),
        "wdl.weight": _bf16(model.wdl_head.weight),
        "wdl.bias": _bf16(model.wdl_head.bias),
        "moves_left.weight": _bf16(model.moves_left_head.weight),
        "moves_left.bias": _bf16(model.moves_left_head.bias),
    }


def build_model(config: ModelConfig) -> DenseChessNet | Moe64A2ChessNet:
    """src/chess_engine_4/model/registry.py:39-44."""

    if isinstance(config, DenseChessNetConfig):
        return DenseChessNet(config)
    if isinstance(config, Moe64A2ChessNetConfig):
        return Moe64A2ChessNet(config)
    raise TypeError(f"unsupported model config type: {type(config).__name__}")


def model_parameter_count(config: ModelConfig) -> int:
    if isinstance(config, DenseChessNetConfig):
        return dense_parameter_count(
            history_length=config.history_length,
            d_model=config.d_model,
            depth=config.depth,
            expansion_ratio=config.expansion_ratio,
            activation=config.activation,
        )
    if isinstance(config, Moe64A2ChessNetConfig):
        return moe64a2_parameter_count(
            history_length=config.history_length,
            d_model=config.d_model,
            depth=config.depth,
            expansion_ratio=config.expansion_ratio,
        )
    raise TypeError(f"unsupported model config type: {type(config).__name__}")
