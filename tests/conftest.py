"""Test configuration: the `gpu` marker and import paths for the package and oracle."""

from __future__ import annotations

import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
for path in (REPO / "chess-engine-4_b200", REPO):
    if str(path) not in sys.path:
        sys.path.insert(0, str(path))


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def pytest_collection_modifyitems(config: pytest.Config, items: list[pytest.Item]) -> None:
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(autouse=True)
def _device_error_word_stays_clear(request: pytest.FixtureRequest):
    """GPU tests must not leave a bounded in-kernel wait timed out."""

    yield
    if "gpu" not in request.keywords:
        return
    import torch

    if not torch.cuda.is_available():
        return
    from ce4b200 import _lib

    code = _lib.check_device_error(torch.cuda.current_device())
    assert code == 0, f"a kernel wait timed out (device error code {code})"
