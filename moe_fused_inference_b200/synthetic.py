"""Seeded synthetic workload pieces shared by the benchmark and the tests.

The reference measures nothing on a public dataset for this path; its
benchmark configurations are random-init models.  ``zipf_bias`` is the load
skew of the prefill and expert-parallel configurations: a Zipf(s) per-expert
logit bias added to the router logits before top-k, so that a few experts
receive many more tokens than the rest.
"""

from __future__ import annotations

import numpy as np


def zipf_bias(n_experts: int, alpha: float, s: float = 1.2, seed: int = 0) -> np.ndarray:
    """Per-expert logit bias ``alpha * log(1 / rank^s)`` (float32, shape (E,)),
    the ranks 1..E assigned to the experts by a seeded permutation."""
    rank = np.random.default_rng(seed).permutation(n_experts) + 1
    return (alpha * -s * np.log(rank)).astype(np.float32)
