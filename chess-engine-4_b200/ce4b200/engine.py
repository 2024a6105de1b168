"""Engine-facing API: Safetensors v1 export and the host-buffer evaluator.

* ``exported_model`` / ``export_model`` write the weight file the reference's release
  exporter writes (src/chess_engine_4/release/export.py:53-57, 60-162, metadata
  :191-219), from a ``DenseChessNet`` / ``Moe64A2ChessNet`` or a Safetensors-named dict.
* ``Engine`` mirrors ``chess_engine_4::inference::Model`` (kernels/include/chess_engine_4/
  inference.h:29-51): ``Engine.load(path, gpu, max_batch)`` then ``evaluate(planes)`` with
  lc0 ``InputPlane`` records on the host, returning policy logits, WDL probabilities and
  moves-left as host arrays. ``evaluate_async`` is the stream-ordered form; consecutive
  calls on different streams overlap one call's copies with the other's forward.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from pathlib import Path

import torch

from . import _lib

FORMAT_NAME = "chess-engine-4"
FORMAT_VERSION = "1"
INPUT_PLANE_COUNT = 112
BOARD_SIZE = 8
POLICY_SIZE = 1858


def safetensors_metadata(
    *,
    architecture: str,
    d_model: int,
    depth: int,
    expansion_ratio: float,
    history_length: int = 8,
    rms_norm_eps: float = 1e-6,
    policy_storage_size: int = 1888,
    source_run: str = "",
    source_step: str = "",
) -> dict[str, str]:
    """String metadata of a Safetensors v1 model file (export.py:191-219, MoE keys
    :153-160)."""

    if architecture not in ("dense", "moe64a2"):
        raise ValueError(f"Safetensors export does not support architecture {architecture!r}.")
    meta = {
        "format": FORMAT_NAME,
        "format_version": FORMAT_VERSION,
        "architecture": architecture,
        "d_model": str(int(d_model)),
        "depth": str(int(depth)),
        "expansion_ratio": str(float(expansion_ratio)),
        "activation": "swiglu",
        "history_length": str(int(history_length)),
        "input_planes": str(INPUT_PLANE_COUNT),
        "board_size": str(BOARD_SIZE),
        "policy_size": str(POLICY_SIZE),
        "policy_storage_size": str(int(policy_storage_size)),
        "wdl_size": "3",
        "moves_left_size": "1",
        "rms_norm_eps": str(float(rms_norm_eps)),
        "input_format": "lc0-classical-112",
        "input_normalization": "history-select-rule50-div99-v1",
        "source_run": source_run,
        "source_step": source_step,
    }
    if architecture == "moe64a2":
        meta.update({"num_experts": "64", "num_active_experts": "2", "layer_pattern": "alternating-moe-dense"})
    return meta


def exported_model(model) -> tuple[dict[str, torch.Tensor], dict[str, str]]:
    """(tensors, metadata) of a ``DenseChessNet`` / ``Moe64A2ChessNet`` (export.py:60-72)."""

    cfg = model.config
    arch = "moe64a2" if type(model).__name__ == "Moe64A2ChessNet" else "dense"
    tensors = {k: v.detach().to("cpu").contiguous() for k, v in model.safetensors_tensors().items()}
    meta = safetensors_metadata(
        architecture=arch,
        d_model=cfg.d_model,
        depth=cfg.depth,
        expansion_ratio=cfg.expansion_ratio,
        history_length=cfg.history_length,
        rms_norm_eps=cfg.rms_norm_eps,
        policy_storage_size=int(tensors["policy.weight"].shape[0]),
    )
    return tensors, meta


def export_model(model, output_path: str | Path) -> None:
    """Writes ``model`` as a Safetensors v1 file (export.py:53-57)."""

    from safetensors.torch import save_file

    tensors, meta = exported_model(model)
    path = Path(output_path)
    path.parent.mkdir(parents=True, exist_ok=True)
    save_file(tensors, str(path), metadata=meta)


@dataclass(frozen=True)
class EngineInfo:
    d_model: int
    depth: int
    history_length: int
    policy_size: int
    maximum_batch_size: int


class Engine:
    """One model on one GPU behind the C ABI (``ce4b_model_load_safetensors``)."""

    def __init__(self, handle: ctypes.c_void_p, device: int) -> None:
        self.lib = _lib.library()
        self.handle = handle
        self.device = device
        info = _lib.ModelInfoStruct()
        _lib.check(self.lib.ce4b_model_info_get(handle, ctypes.byref(info)))
        self.info = EngineInfo(info.d_model, info.depth, info.history_length, info.policy_size,
                               info.maximum_batch_size)

    @classmethod
    def load(cls, path: str | Path, gpu: int = 0, max_batch: int = 1024, precision: str = "bf16") -> "Engine":
        """Model::Load (inference.h:31-33): reads and validates the file, uploads the
        weights, plans the workspace for ``max_batch`` positions."""

        if precision not in ("bf16", "mxfp8"):
            raise ValueError(f"unsupported precision {precision!r}")
        lib = _lib.library()
        handle = ctypes.c_void_p()
        _lib.check(lib.ce4b_model_load_safetensors(
            str(path).encode(), gpu, max_batch,
            _lib.PRECISION_BF16 if precision == "bf16" else _lib.PRECISION_MXFP8, ctypes.byref(handle)))
        return cls(handle, gpu)

    @staticmethod
    def _check_planes(planes: torch.Tensor) -> int:
        """``planes`` holds 16-byte InputPlane records {u64 mask; f32 value; u32 pad}:
        int64 [B, 112, 2] (as ``synthetic.lc0_planes_tensor`` makes) or int32 [B, 112, 4]."""

        words = {torch.int64: 2, torch.int32: 4}.get(planes.dtype)
        if planes.device.type != "cpu" or words is None or planes.dim() != 3 or tuple(planes.shape[1:]) != (
            INPUT_PLANE_COUNT, words
        ):
            raise ValueError("planes must be a CPU tensor of InputPlane records, int64 [B, 112, 2] or int32 [B, 112, 4]")
        if not planes.is_contiguous():
            raise ValueError("planes must be contiguous")
        return int(planes.shape[0])

    def outputs(self, batch: int, pin: bool = True) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """Host output buffers for ``batch`` positions (pinned by default)."""

        def empty(*shape: int) -> torch.Tensor:
            t = torch.empty(*shape, dtype=torch.float32)
            return t.pin_memory() if pin else t

        return empty(batch, self.info.policy_size), empty(batch, 3), empty(batch)

    def evaluate(self, planes: torch.Tensor, out=None) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """Model::Evaluate (inference.h:35-40): blocking; returns (policy logits [B,1858],
        WDL probabilities [B,3], moves-left [B])."""

        batch = self._check_planes(planes)
        policy, wdl, ml = out if out is not None else self.outputs(batch, pin=False)
        _lib.check(self.lib.ce4b_model_evaluate(self.handle, planes.data_ptr(), batch, policy.data_ptr(),
                                                wdl.data_ptr(), ml.data_ptr()))
        return policy, wdl, ml

    def set_direct_io(self, enabled: bool) -> None:
        """Copy-free small-batch evaluation of pinned host buffers (on by default): the
        expansion kernel reads the records and the heads write the outputs in place."""

        _lib.check(self.lib.ce4b_model_set_direct_io(self.handle, 1 if enabled else 0))

    def evaluate_async(self, planes: torch.Tensor, out, stream: torch.cuda.Stream) -> None:
        """Enqueues the evaluation on ``stream``; ``planes`` and ``out`` must be pinned and
        stay untouched until the stream reaches this point."""

        batch = self._check_planes(planes)
        policy, wdl, ml = out
        _lib.check(self.lib.ce4b_model_evaluate_async(self.handle, planes.data_ptr(), batch, policy.data_ptr(),
                                                      wdl.data_ptr(), ml.data_ptr(), stream.cuda_stream))

    def evaluate_legal(
        self, planes: torch.Tensor, move_offsets: torch.Tensor, move_indices: torch.Tensor,
        temperature: float = 1.0,
    ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """Legal-move probabilities instead of the full policy (the lc0 backend's
        post-processing on the GPU): returns (probs [nnz], wdl probabilities [B, 3],
        moves-left [B]); move_offsets int32 [B + 1], move_indices int32 [nnz]."""

        batch = self._check_planes(planes)
        offsets = move_offsets.to(torch.int32).contiguous()
        indices = move_indices.to(torch.int32).contiguous()
        if offsets.shape != (batch + 1,) or int(offsets[-1]) != indices.numel():
            raise ValueError("move_offsets must be [B + 1] ending at len(move_indices)")
        probs = torch.empty(indices.numel(), dtype=torch.float32)
        wdl = torch.empty(batch, 3, dtype=torch.float32)
        ml = torch.empty(batch, dtype=torch.float32)
        _lib.check(self.lib.ce4b_model_evaluate_legal(
            self.handle, planes.data_ptr(), batch, offsets.data_ptr(), indices.data_ptr(),
            float(temperature), probs.data_ptr(), wdl.data_ptr(), ml.data_ptr()))
        return probs, wdl, ml

    def close(self) -> None:
        if self.handle is not None and self.handle.value:
            self.lib.ce4b_model_destroy(self.handle)
            self.handle = None

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:
            pass
