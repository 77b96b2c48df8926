"""Route-id generators with the semantics of the reference's make_route_ids
(include/raggedroute/benchmark/adapter_utils.h:206-248): per token, top_k
ids; "uniform" and "zipf" draw without repeats inside a token, "single_hot"
gives rank r expert r, "round_robin" (token + rank) % E, "duplicate_route"
sends every route to expert 0. Seeded numpy generators stand in for the
reference's std::mt19937_64 (the oracle receives the same ids)."""
from __future__ import annotations

import numpy as np


def make_route_ids(tokens: int, top_k: int, experts: int, distribution: str,
                   zipf_s: float = 1.0, seed: int = 0) -> np.ndarray:
    if tokens < 1 or top_k < 1 or experts < top_k:
        raise ValueError("route shape requires tokens>=1 and experts>=top_k>=1")
    rng = np.random.default_rng(seed)
    ids = np.empty((tokens, top_k), np.int32)
    if distribution == "duplicate_route":
        ids[:] = 0
    elif distribution == "single_hot":
        ids[:] = np.arange(top_k, dtype=np.int32)[None, :]
    elif distribution == "round_robin":
        ids[:] = (np.arange(tokens)[:, None] + np.arange(top_k)[None, :]) % experts
    elif distribution in ("uniform", "zipf"):
        p = np.ones(experts) if distribution == "uniform" else \
            np.power(np.arange(1, experts + 1, dtype=np.float64), -zipf_s)
        p = p / p.sum()
        for t in range(tokens):
            ids[t] = rng.choice(experts, size=top_k, replace=False, p=p)
    else:
        raise ValueError(f"unsupported distribution: {distribution}")
    return ids


def make_route_weights(tokens: int, top_k: int, seed: int = 0) -> np.ndarray:
    """U(0.01, 1) per route, normalised per token
    (postroute_chain_adapter.cpp:684-694)."""
    rng = np.random.default_rng(seed + 1)
    w = rng.uniform(0.01, 1.0, (tokens, top_k)).astype(np.float32)
    return (w / w.sum(axis=1, keepdims=True)).astype(np.float32)
