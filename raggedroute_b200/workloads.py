"""Seeded synthetic inputs with the shapes and value distributions of the five
BASELINE configurations (C1-C5). The reference's inputs are synthetic too
(include/raggedroute/benchmark/adapter_utils.h:197-248); no dataset is
involved. "N(0, s)" means standard deviation s. Large tensors are generated
on the target device with a seeded torch.Generator; small integer structures
(group sizes, tie/NaN rows) with numpy.
"""
from __future__ import annotations

import dataclasses
import math

import numpy as np
import torch

C1 = dict(name="C1", tokens=512, hidden=256, experts=32, output=64, seed=0)
C2 = dict(name="C2", tokens=4096, hidden=256, experts=64, output=128, seed=1)
C3 = dict(name="C3", routes=1 << 20, hidden=128, experts=(1, 8, 64, 256), seed=2)
C4 = dict(name="C4", routes=32768, hidden=1024, experts=64, output=1024, seed=3, empty=6)
C5 = dict(name="C5", tokens=65536, hidden=4096, experts=128, output=1408, seed=4)


def _gen(device, seed: int) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def uniform(shape, seed: int, device="cpu", low=-1.0, high=1.0) -> torch.Tensor:
    g = _gen(device, seed)
    return torch.rand(shape, generator=g, device=device, dtype=torch.float32) * (high - low) + low


def normal(shape, std: float, seed: int, device="cpu") -> torch.Tensor:
    g = _gen(device, seed)
    return torch.randn(shape, generator=g, device=device, dtype=torch.float32) * std


def zipf_log_bias(experts: int, s: float) -> np.ndarray:
    """log p_e with p_e proportional to (e+1)^-s, normalised."""
    p = np.power(np.arange(1, experts + 1, dtype=np.float64), -s)
    p /= p.sum()
    return np.log(p).astype(np.float32)


@dataclasses.dataclass
class ChainInputs:
    x: torch.Tensor
    router_w: torch.Tensor | None
    logit_bias: torch.Tensor | None
    expert_w: torch.Tensor
    logits: torch.Tensor | None = None


def c1_inputs(device="cpu") -> ChainInputs:
    """chain_from_tokens, T=512 K=256 E=32 N=64, seed 0."""
    t, k, e, n, s = C1["tokens"], C1["hidden"], C1["experts"], C1["output"], C1["seed"]
    return ChainInputs(x=uniform((t, k), s * 10 + 1, device),
                       router_w=normal((k, e), 1.0 / math.sqrt(k), s * 10 + 2, device),
                       logit_bias=None,
                       expert_w=normal((e, k, n), 1.0 / math.sqrt(k), s * 10 + 3, device))


def c2_logits(tokens: int = 4096, experts: int = 64, seed: int = 1) -> np.ndarray:
    """Logits ~ N(0,1) + log-Zipf(1.2) bias; every 32nd row carries an exact
    top-1/top-2 tie; every 1024th row holds one NaN."""
    rng = np.random.default_rng(seed)
    logits = rng.standard_normal((tokens, experts)).astype(np.float32)
    logits += zipf_log_bias(experts, 1.2)[None, :]
    for t in range(0, tokens, 32):
        row = logits[t]
        order = np.argsort(-row, kind="stable")
        row[order[1]] = row[order[0]]
    for t in range(0, tokens, 1024):
        logits[t, rng.integers(0, experts)] = np.nan
    return logits


def c2_inputs(device="cpu") -> ChainInputs:
    """chain_from_logits, T=4096 E=64 K=256 N=128, seed 1."""
    t, k, e, n, s = C2["tokens"], C2["hidden"], C2["experts"], C2["output"], C2["seed"]
    return ChainInputs(x=uniform((t, k), s * 10 + 1, device), router_w=None, logit_bias=None,
                       expert_w=normal((e, k, n), 1.0 / math.sqrt(k), s * 10 + 3, device),
                       logits=torch.from_numpy(c2_logits(t, e, s)).to(device))


def route_ids(routes: int, experts: int, dist: str, seed: int, s: float = 1.5) -> np.ndarray:
    """C3 route ids: 'uniform', 'zipf' (s, drawn per route) or 'one' (all 0)."""
    rng = np.random.default_rng(seed)
    if dist == "uniform":
        return rng.integers(0, experts, routes, dtype=np.int32)
    if dist == "zipf":
        p = np.power(np.arange(1, experts + 1, dtype=np.float64), -s)
        p /= p.sum()
        return rng.choice(experts, size=routes, p=p).astype(np.int32)
    if dist == "one":
        return np.zeros(routes, np.int32)
    raise ValueError(dist)


def c4_group_sizes(routes: int = 32768, experts: int = 64, empty: int = 6, s: float = 1.1,
                   seed: int = 3) -> np.ndarray:
    """Zipf(1.1) group sizes over experts-empty experts, `empty` seeded
    forced-empty experts, every non-empty size not a multiple of 16, sum = routes."""
    rng = np.random.default_rng(seed)
    empty_ids = rng.choice(experts, size=empty, replace=False)
    active = np.array([e for e in range(experts) if e not in set(empty_ids.tolist())])
    ranks = rng.permutation(len(active))
    p = np.power(ranks + 1.0, -s)
    p /= p.sum()
    sizes = np.zeros(experts, np.int64)
    sizes[active] = np.maximum(1, np.floor(p * routes)).astype(np.int64)
    sizes[active[0]] += routes - sizes.sum()
    # Move single rows until no active size is a multiple of 16.
    for _ in range(10 * experts):
        bad = [e for e in active if sizes[e] % 16 == 0]
        if not bad:
            break
        e = bad[0]
        donor = max(active, key=lambda d: sizes[d] if d != e else -1)
        sizes[e] += 1
        sizes[donor] -= 1
    assert sizes.sum() == routes and all(sizes[e] % 16 != 0 for e in active)
    return sizes.astype(np.int32)


def offsets_from_sizes(sizes: np.ndarray) -> np.ndarray:
    return np.concatenate([[0], np.cumsum(sizes)]).astype(np.int32)


def c5_inputs(device="cuda", tokens: int | None = None, rank: int = 0) -> ChainInputs:
    """Expert-parallel chain_from_tokens, T=65536 K=4096 E=128 N=1408, seed 4,
    router logits biased by log-Zipf(1.0) per expert. Each rank of a
    multi-GPU run draws its own token batch (seed offset by rank); the
    weights are shared."""
    t = tokens or C5["tokens"]
    k, e, n, s = C5["hidden"], C5["experts"], C5["output"], C5["seed"]
    return ChainInputs(x=normal((t, k), 1.0, s * 10 + 1 + 1000 * rank, device),
                       router_w=normal((k, e), 1.0 / math.sqrt(k), s * 10 + 2, device),
                       logit_bias=torch.from_numpy(zipf_log_bias(e, 1.0)).to(device),
                       expert_w=normal((e, k, n), 1.0 / math.sqrt(k), s * 10 + 3, device))
