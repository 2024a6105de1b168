"""The header-only chess_engine_4::inference facade (include/chess_engine_4/inference.h):
compiles as C++20 (CPU), and on the GPU gives exactly the C ABI engine's outputs."""

from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest
import torch

REPO = Path(__file__).resolve().parents[1]
MAIN = REPO / "tests" / "cpp" / "inference_facade_main.cpp"
LIBDIR = REPO / "chess-engine-4_b200" / "ce4b200"


def _compile(out: Path, syntax_only: bool = False) -> None:
    cxx = shutil.which("g++")
    if cxx is None:
        pytest.skip("g++ not available")
    cmd = [cxx, "-std=c++20", "-O1", "-I", str(REPO / "include"), str(MAIN)]
    if syntax_only:
        cmd += ["-fsyntax-only"]
    else:
        cmd += ["-o", str(out), "-L", str(LIBDIR), "-lce4b200", f"-Wl,-rpath,{LIBDIR}"]
    subprocess.run(cmd, check=True, capture_output=True, text=True)


def test_facade_header_compiles_as_cpp20(tmp_path) -> None:
    _compile(tmp_path / "unused", syntax_only=True)
    _compile(tmp_path / "facade")  # and links against libce4b200.so (no GPU needed)


@pytest.mark.gpu
def test_facade_evaluate_equals_engine(tmp_path) -> None:
    from ce4b200 import DenseChessNet, DenseChessNetConfig, Engine, export_model, synthetic

    model = DenseChessNet(DenseChessNetConfig(d_model=128, depth=2, expansion_ratio=3.0))
    synthetic.load_into(model, synthetic.make_dense_weights(d_model=128, depth=2, hidden_dim=384, seed=3))
    path = tmp_path / "m.safetensors"
    export_model(model, path)
    batch = 96
    planes = synthetic.lc0_planes_tensor(synthetic.make_lc0_planes(batch, 12))
    planes.numpy().astype(np.int64).tofile(tmp_path / "planes.bin")
    exe = tmp_path / "facade"
    _compile(exe)
    run = subprocess.run([str(exe), str(path), str(tmp_path / "planes.bin"), str(batch), str(tmp_path / "out.bin")],
                         capture_output=True, text=True, timeout=300)
    assert run.returncode == 0, run.stderr
    out = np.fromfile(tmp_path / "out.bin", dtype=np.float32)
    engine = Engine.load(path, gpu=0, max_batch=batch)
    policy, wdl, ml = engine.evaluate(planes)
    ps = policy.shape[1]
    assert np.array_equal(out[: batch * ps].reshape(batch, ps), policy.numpy())
    assert np.array_equal(out[batch * ps: batch * ps + batch * 3].reshape(batch, 3), wdl.numpy())
    assert np.array_equal(out[batch * ps + batch * 3:], ml.numpy())
    assert torch.isfinite(policy).all()
