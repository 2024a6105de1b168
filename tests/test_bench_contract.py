"""bench.py's reference arm runs on the host cores (no GPU) and prints the one JSON line of
the benchmark contract: check its keys and their types on the smallest configuration."""

from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]


def test_reference_arm_prints_contract_line() -> None:
    out = subprocess.run(
        [sys.executable, str(REPO / "bench.py"), "--impl", "reference", "--config", "c0", "--steps", "1",
         "--warmup", "1"],
        cwd=REPO, capture_output=True, text=True, timeout=600, check=True,
    )
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, out.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    for key in ("metric", "unit", "dtype", "data", "scaling"):
        assert isinstance(d[key], str) and d[key]
    assert d["value"] > 0 and d["ms_per_step"] > 0
    assert d["n_gpus"] == 1 and d["steps"] == 1 and d["warmup"] == 1
    assert d["higher_is_better"] is True
    assert "vs_baseline" in d
    assert d["config"]["workload"].startswith("dense-d128-L6")
    cpu = d["cpu_baseline"]
    assert cpu["kind"] in ("port", "reference") and cpu["cores"] >= 1 and cpu["sample"]
    assert cpu["value"] == d["value"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


@pytest.mark.gpu
def test_our_arm_prints_roofline_and_launch_count() -> None:
    out = subprocess.run(
        [sys.executable, str(REPO / "bench.py"), "--quick", "--config", "c0", "--steps", "3", "--warmup", "3"],
        cwd=REPO, capture_output=True, text=True, timeout=900, check=True,
    )
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, out.stdout
    d = json.loads(lines[0])
    assert "impl" not in d and d["value"] > 0 and d["n_gpus"] == 1
    roof = d["roofline"]
    assert roof["bound"] in ("tensor", "hbm") and roof["unit"] in ("TFLOP/s", "GB/s")
    assert roof["achieved"] > 0 and roof["peak"] > 0
    assert abs(roof["frac"] - roof["achieved"] / roof["peak"]) < 1e-6
    assert d["gpu_launches"] > 0 and d["kernels_per_step"] >= 1
    assert "dense_tower" in d["kernel_ms_per_step"]
