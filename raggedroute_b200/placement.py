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


class ReplicatedPlacement:
    """Virtual-expert placement for the EP runtime.

    Every real expert e gets r_e = clamp(ceil(load_e / fair_share), 1, G)
    replicas ("virtual experts"); replica j serves the source ranks s with
    (s * r_e) // G == j, so a hot expert's tokens are split by source rank.
    Virtual experts are placed by LPT under the runtime's constraint that every
    rank owns the same number of them (zero-load padding entries fill up), with
    replicas of one expert kept on distinct ranks when possible, and then
    numbered rank by rank so each rank's virtual ids are contiguous.

    Attributes: virtual_experts (V, a multiple of nranks), virtual_to_real [V]
    (padding entries point at real expert 0 and are never routed to),
    remap [nranks, R] (real id -> virtual id for routes from source rank s),
    rank_load [nranks] (expected load per rank).
    """

    def __init__(self, loads, nranks: int, max_virtual: int = 1024):
        loads = np.asarray(loads, dtype=np.float64)
        r_experts = loads.size
        total = float(loads.sum())
        fair = total / nranks if total > 0 else 1.0
        reps = np.clip(np.ceil(loads / fair - 1e-9), 1, nranks).astype(np.int64)
        items = []  # (load, real expert, replica index)
        for e in range(r_experts):
            r = int(reps[e])
            for j in range(r):
                n_src = sum(1 for s in range(nranks) if (s * r) // nranks == j)
                items.append((loads[e] * n_src / nranks, e, j))
        pad = (-len(items)) % nranks
        items += [(0.0, -1, 0)] * pad
        v_count = len(items)
        if v_count > max_virtual:
            raise ValueError("too many virtual experts")
        per = v_count // nranks
        rank_load = np.zeros(nranks)
        slots = np.full(nranks, per)
        hosts: dict[int, set] = {}
        rank_of_item = np.empty(v_count, dtype=np.int64)
        for i in sorted(range(v_count), key=lambda i: -items[i][0]):
            load, e, _ = items[i]
            free = [r for r in range(nranks) if slots[r] > 0]
            avoid = hosts.get(e, set()) if e >= 0 else set()
            pool = [r for r in free if r not in avoid] or free
            r = min(pool, key=lambda q: rank_load[q])
            rank_of_item[i] = r
            rank_load[r] += load
            slots[r] -= 1
            if e >= 0:
                hosts.setdefault(e, set()).add(r)
        order = sorted(range(v_count), key=lambda i: (rank_of_item[i], i))
        self.nranks = nranks
        self.router_experts = r_experts
        self.virtual_experts = v_count
        self.replicas = reps
        self.virtual_to_real = np.zeros(v_count, dtype=np.int64)
        replica_vid = {}
        for v, i in enumerate(order):
            _, e, j = items[i]
            self.virtual_to_real[v] = max(e, 0)
            if e >= 0:
                replica_vid[(e, j)] = v
        self.remap = np.zeros((nranks, r_experts), dtype=np.int32)
        for s in range(nranks):
            for e in range(r_experts):
                self.remap[s, e] = replica_vid[(e, (s * int(reps[e])) // nranks)]
        self.rank_load = rank_load

    def imbalance(self) -> float:
        return float(self.rank_load.max() / self.rank_load.mean())
