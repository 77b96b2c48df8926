"""raggedroute_b200 -- B200-native RaggedRoute routing path.

The product is ``libraggedroute_b200.so`` (C ABI declared in
``include/raggedroute_b200.h``; reference-compatible C++ API in
``include/raggedroute/``). This package is the Python host binding over that C
ABI, used by the tests, the benchmark and Python callers. Device memory and
streams come from PyTorch; every operator call goes through the C ABI into the
sm_100a kernels. There is no CPU or PyTorch fallback: if the library is
missing or fails to load, every call raises.

Operator names, argument meaning and status codes follow RaggedRoute's v0.2
operator API (include/raggedroute/operators.h:114-135 of the reference).
"""
from __future__ import annotations

from raggedroute_b200._lib import (  # noqa: F401
    ARCH_AUTO,
    ARCH_OTHER,
    ARCH_SM86,
    ARCH_SM90,
    ARCH_SM100,
    FAMILY_AUTO,
    FAMILY_CUDA_NAIVE,
    FAMILY_CUDA_OPTIMIZED,
    MAX_EXPERTS,
    StatusCode,
    RaggedRouteError,
    Context,
    lib,
    library_path,
)
from raggedroute_b200.ops import (  # noqa: F401
    dense_gemm,
    topk_gate,
    topk_gate_biased,
    histogram,
    exclusive_scan,
    histogram_exclusive_scan,
    token_permute,
    token_permute_workspace_size,
    grouped_gemm,
    grouped_gemm_gather,
    grouped_gemm_combine,
    grouped_gemm_scatter,
    grouped_gemm_prepared,
    PreparedExpertWeights,
    unpermute,
    chain_from_tokens,
    chain_from_logits,
    chain_workspace_size,
    ChainBuffers,
    RouteChainBuffers,
    chain_from_route_ids,
    HostChain,
    Graph,
    kernel_launch_count,
    grouped_gemm_engine,
)

__all__ = [
    "dense_gemm", "topk_gate", "histogram", "exclusive_scan", "histogram_exclusive_scan",
    "token_permute", "grouped_gemm", "unpermute", "chain_from_tokens", "chain_from_logits",
    "chain_from_route_ids",
    "HostChain", "Context", "RaggedRouteError", "StatusCode", "lib",
]
