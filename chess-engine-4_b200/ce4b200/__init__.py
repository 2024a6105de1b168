"""ce4b200 — B200 (sm_100a) forward path for the chess-engine-4 networks.

Public API mirrors ``chess_engine_4.model`` (model classes, configs, output type) and
``chess_engine_4.kernels`` (kernel operators); computation runs in libce4b200.so.
"""

from .engine import Engine, export_model, exported_model, safetensors_metadata
from .model import (
    ChessNetOutput,
    DenseChessNet,
    DenseChessNetConfig,
    Moe64A2ChessNet,
    Moe64A2ChessNetConfig,
    build_model,
    dense_parameter_count,
    model_config_from_dict,
    model_parameter_count,
    moe64a2_parameter_count,
    normalize_lc0_planes,
    select_lc0_history,
)

__all__ = [
    "ChessNetOutput",
    "Engine",
    "export_model",
    "exported_model",
    "safetensors_metadata",
    "DenseChessNet",
    "DenseChessNetConfig",
    "Moe64A2ChessNet",
    "Moe64A2ChessNetConfig",
    "build_model",
    "dense_parameter_count",
    "model_config_from_dict",
    "model_parameter_count",
    "moe64a2_parameter_count",
    "normalize_lc0_planes",
    "select_lc0_history",
]
