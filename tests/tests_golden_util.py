"""Helpers shared by the golden-fixture generator and the tests."""

from __future__ import annotations

import hashlib

import torch


def weight_checksum(weights: dict[str, torch.Tensor]) -> str:
    """SHA-256 over the sorted tensor names and their raw bytes."""

    h = hashlib.sha256()
    for name in sorted(weights):
        h.update(name.encode())
        h.update(weights[name].contiguous().view(torch.uint8).numpy().tobytes())
    return h.hexdigest()
