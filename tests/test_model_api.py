"""The drop-in model API mirrors the reference's (config checks, parameter names, counts)
without needing a GPU."""

from __future__ import annotations

import pytest
import torch


def test_config_validation_matches_reference_messages() -> None:
    from ce4b200 import DenseChessNetConfig, Moe64A2ChessNetConfig, model_config_from_dict

    with pytest.raises(ValueError, match="at least 64"):
        DenseChessNetConfig(d_model=32)
    with pytest.raises(ValueError, match="history_length"):
        DenseChessNetConfig(history_length=9)
    with pytest.raises(ValueError, match="positive even"):
        Moe64A2ChessNetConfig(d_model=64, depth=3)
    with pytest.raises(ValueError, match="unknown key"):
        model_config_from_dict({"kind": "moe64a2", "num_experts": 32})
    with pytest.raises(ValueError, match="policy_size"):
        model_config_from_dict({"policy_size": 100})
    cfg = model_config_from_dict({"kind": "moe64a2", "d_model": 64, "depth": 2, "expansion_ratio": 2.0})
    assert isinstance(cfg, Moe64A2ChessNetConfig)
    assert cfg.num_experts == 64 and cfg.num_active_experts == 2
    assert Moe64A2ChessNetConfig(d_model=512).cuda_graph_compatible
    assert not Moe64A2ChessNetConfig(d_model=1024).cuda_graph_compatible


def test_parameter_counts_match_reference_known_answers() -> None:
    from ce4b200 import dense_parameter_count, moe64a2_parameter_count

    # tests/test_model_and_losses.py:215-220 and :64-68 of the reference.
    assert moe64a2_parameter_count(d_model=64, depth=2, expansion_ratio=2.0) == 2_212_000
    full = dense_parameter_count(d_model=64, depth=2, history_length=8)
    short = dense_parameter_count(d_model=64, depth=2, history_length=2)
    assert full - short == (8 - 2) * 13 * 64 * 64


def test_dense_module_state_dict_uses_transformer_engine_names() -> None:
    from ce4b200 import DenseChessNet, DenseChessNetConfig, dense_parameter_count

    model = DenseChessNet(DenseChessNetConfig(d_model=64, depth=2, expansion_ratio=3.0, precision="bf16"))
    names = set(model.state_dict())
    expected = {
        "input.weight", "input.bias", "norm.weight",
        "policy_head.weight", "policy_head.bias", "wdl_head.weight", "wdl_head.bias",
        "moves_left_head.weight", "moves_left_head.bias",
        "blocks.0.layer.layer_norm_weight", "blocks.0.layer.fc1_weight", "blocks.0.layer.fc2_weight",
        "blocks.1.layer.layer_norm_weight", "blocks.1.layer.fc1_weight", "blocks.1.layer.fc2_weight",
    }
    assert names == expected
    assert model.policy_head.weight.shape == (1888, 64)
    assert model.blocks[0].layer.fc1_weight.shape == (2 * 192, 64)
    total = sum(p.numel() for p in model.parameters())
    assert total == dense_parameter_count(d_model=64, depth=2, expansion_ratio=3.0, activation="swiglu")
    assert all(p.dtype == torch.bfloat16 for p in model.parameters())


def test_moe_module_names_and_count() -> None:
    from ce4b200 import Moe64A2ChessNet, Moe64A2ChessNetConfig, moe64a2_parameter_count

    model = Moe64A2ChessNet(Moe64A2ChessNetConfig(d_model=64, depth=2, expansion_ratio=2.0, precision="bf16"))
    names = set(model.state_dict())
    assert "blocks.0.router.weight" in names and "blocks.0.router_qb_beta" in names
    assert "blocks.0.experts.0.weight63" in names and "blocks.0.experts.2.weight0" in names
    assert "blocks.1.layer.fc1_weight" in names
    params = sum(p.numel() for p in model.parameters())
    assert params == moe64a2_parameter_count(d_model=64, depth=2, expansion_ratio=2.0)
    tensors = model.safetensors_tensors()
    assert tensors["blocks.0.experts.gate_up.weight"].shape == (64, 256, 64)
    assert tensors["blocks.0.experts.down.weight"].shape == (64, 64, 128)
    assert tensors["blocks.0.router_qb_beta"].dtype == torch.float32


def test_safetensors_names_follow_export_contract() -> None:
    from ce4b200 import DenseChessNet, DenseChessNetConfig

    model = DenseChessNet(DenseChessNetConfig(d_model=64, depth=1, expansion_ratio=2.0))
    t = model.safetensors_tensors()
    assert set(t) == {
        "input.weight", "input.bias", "final_norm.weight", "policy.weight", "policy.bias",
        "wdl.weight", "wdl.bias", "moves_left.weight", "moves_left.bias",
        "blocks.0.norm.weight", "blocks.0.gate_up.weight", "blocks.0.down.weight",
    }


def test_exported_file_carries_loader_metadata(tmp_path) -> None:
    """The exported file has the metadata the C++ loader validates (keys and values of
    src/chess_engine_4/release/export.py:191-219, MoE keys :153-160)."""

    from safetensors import safe_open

    from ce4b200 import DenseChessNet, DenseChessNetConfig, Moe64A2ChessNet, Moe64A2ChessNetConfig, export_model

    dense = DenseChessNet(DenseChessNetConfig(d_model=64, depth=2, expansion_ratio=3.0))
    export_model(dense, tmp_path / "d.safetensors")
    with safe_open(str(tmp_path / "d.safetensors"), "pt") as f:
        meta = f.metadata()
        assert set(f.keys()) == set(dense.safetensors_tensors())
        assert f.get_tensor("policy.weight").dtype == torch.bfloat16
    assert meta["format"] == "chess-engine-4" and meta["format_version"] == "1"
    assert meta["architecture"] == "dense" and meta["activation"] == "swiglu"
    assert (meta["d_model"], meta["depth"], meta["expansion_ratio"]) == ("64", "2", "3.0")
    assert meta["input_format"] == "lc0-classical-112"
    assert meta["input_normalization"] == "history-select-rule50-div99-v1"
    assert (meta["input_planes"], meta["board_size"], meta["policy_size"]) == ("112", "8", "1858")
    assert meta["policy_storage_size"] == "1888" and meta["rms_norm_eps"] == "1e-06"
    assert "num_experts" not in meta

    moe = Moe64A2ChessNet(Moe64A2ChessNetConfig(d_model=64, depth=2, expansion_ratio=1.0))
    export_model(moe, tmp_path / "m.safetensors")
    with safe_open(str(tmp_path / "m.safetensors"), "pt") as f:
        meta = f.metadata()
        assert f.get_tensor("blocks.0.router_qb_beta").dtype == torch.float32
        assert tuple(f.get_tensor("blocks.0.experts.gate_up.weight").shape) == (64, 128, 64)
    assert meta["architecture"] == "moe64a2"
    assert (meta["num_experts"], meta["num_active_experts"], meta["layer_pattern"]) == (
        "64", "2", "alternating-moe-dense"
    )


def test_forward_rejects_cpu_planes_without_fallback() -> None:
    from ce4b200 import DenseChessNet, DenseChessNetConfig

    model = DenseChessNet(DenseChessNetConfig(d_model=64, depth=1, expansion_ratio=2.0, precision="bf16"))
    with pytest.raises(ValueError, match="CUDA"):
        model(torch.zeros(2, 112, 8, 8))
    with pytest.raises(ValueError, match=r"\[B, 112, 8, 8\]"):
        model(torch.zeros(2, 111, 8, 8))


def test_synthetic_weights_are_deterministic() -> None:
    from ce4b200 import synthetic

    a = synthetic.make_dense_weights(d_model=64, depth=1, hidden_dim=128, seed=5)
    b = synthetic.make_dense_weights(d_model=64, depth=1, hidden_dim=128, seed=5)
    assert all(torch.equal(a[k], b[k]) for k in a)
    beta = synthetic.zipf_router_bias(3)
    assert beta.shape == (64,) and float(beta.max()) < 0
