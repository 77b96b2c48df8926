"""Expert placement for expert parallelism.

The EP runtime gives rank g the contiguous expert ids [g*L, (g+1)*L),
L = E / G. With a skewed router (BASELINE C5 adds a log-Zipf(1.0) bias per
expert) contiguous ranges put the hottest experts on rank 0, so experts are
first placed by longest-processing-time (largest expected load first, onto the
least-loaded rank that still has a free slot) and then relabelled so that each
rank's experts are contiguous. Relabelling permutes the expert axis of the
router weights, the logit bias and the expert weights once at set-up; the
chain then runs unchanged.
"""
from __future__ import annotations

import numpy as np


def lpt_placement(loads, nranks: int) -> np.ndarray:
    """Returns rank_of[e] for every expert, each rank getting exactly E/G
    experts and a near-equal share of the expected load."""
    loads = np.asarray(loads, dtype=np.float64)
    experts = loads.size
    if nranks < 1 or experts % nranks != 0:
        raise ValueError("experts must be a multiple of nranks")
    per = experts // nranks
    rank_load = np.zeros(nranks)
    slots = np.full(nranks, per)
    rank_of = np.empty(experts, dtype=np.int64)
    for e in np.argsort(-loads, kind="stable"):
        free = np.flatnonzero(slots > 0)
        r = free[np.argmin(rank_load[free])]
        rank_of[e] = r
        rank_load[r] += loads[e]
        slots[r] -= 1
    return rank_of


def relabel_permutation(rank_of: np.ndarray) -> np.ndarray:
    """new_to_old[j] = original expert id of new expert j, grouping each
    rank's experts contiguously (rank-major, original order inside a rank)."""
    rank_of = np.asarray(rank_of)
    return np.argsort(rank_of, kind="stable")


def expected_loads_from_bias(bias) -> np.ndarray:
    """Expected per-expert load of a router whose logits are a symmetric random
    part plus `bias`: proportional to exp(bias)."""
    b = np.asarray(bias, dtype=np.float64)
    p = np.exp(b - b.max())
    return p / p.sum()


def imbalance(loads, rank_of, nranks: int) -> float:
    """max rank load / mean rank load (1.0 = perfect balance)."""
    loads = np.asarray(loads, dtype=np.float64)
    per_rank = np.bincount(np.asarray(rank_of), weights=loads, minlength=nranks)
    return float(per_rank.max() / per_rank.mean())
