"""CPU restatement of the lc0 ce4 backend's legal-move policy — TEST INFRASTRUCTURE ONLY.

third_party/lc0/src/neural/backends/ce4/backend.cc:182-195: for each position, gather the
logits of its legal moves, subtract their maximum, exponentiate with the policy
temperature, normalise (a zero total leaves the values unscaled). Computed here in FP64
with the exact exponential (the backend uses FastExp, an approximation of it)."""

from __future__ import annotations

import numpy as np


def legal_move_softmax(policy: np.ndarray, offsets: np.ndarray, indices: np.ndarray,
                       temperature: float) -> np.ndarray:
    policy = np.asarray(policy, dtype=np.float64)
    out = np.zeros(len(indices), dtype=np.float64)
    for b in range(policy.shape[0]):
        lo, hi = int(offsets[b]), int(offsets[b + 1])
        if hi <= lo:
            continue
        logits = policy[b, indices[lo:hi]]
        e = np.exp((logits - logits.max()) * temperature)
        total = e.sum()
        out[lo:hi] = e / total if total > 0 else e
    return out
