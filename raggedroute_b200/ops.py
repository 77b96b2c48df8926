"""Python mirror of RaggedRoute's operator API over the C ABI.

Each function takes CUDA tensors (FP32 / int32, contiguous), checks shapes
and dtypes on the host, and calls the matching ``rr_*`` entry point on the
current torch stream (or ``ctx.stream``). Errors come back as
``RaggedRouteError`` carrying the reference's status code. Names and argument
meaning follow include/raggedroute/operators.h:19-135 of the reference.
"""
from __future__ import annotations

import ctypes
import dataclasses

import torch

from raggedroute_b200._lib import Context, check, lib


def _ptr(t: torch.Tensor | None) -> int | None:
    if t is None:
        return None
    return t.data_ptr() or None


def _ctx(ctx: Context | None, workspace: torch.Tensor | None = None) -> ctypes.POINTER:
    c = dataclasses.replace(ctx) if ctx is not None else Context()
    if c.stream == 0 and torch.cuda.is_available():
        c.stream = torch.cuda.current_stream().cuda_stream
    if workspace is not None:
        c.workspace = workspace.data_ptr()
        c.workspace_bytes = workspace.numel() * workspace.element_size()
    return ctypes.pointer(c.as_c())


CHAIN_IMPL_GATHER_ROWS = 1
CHAIN_IMPL_PREPARED_WEIGHTS = 2
CHAIN_IMPL_FUSED_COMBINE = 4


def _chain_ctx(ctx: Context | None, workspace: torch.Tensor, gather_rows: bool,
               prepared: bool = False, fused_combine: bool = False):
    if gather_rows and prepared:
        raise ValueError("gather_rows does not combine with prepared expert weights")
    c = dataclasses.replace(ctx) if ctx is not None else Context()
    bits = ((CHAIN_IMPL_GATHER_ROWS if gather_rows else 0) |
            (CHAIN_IMPL_PREPARED_WEIGHTS if prepared else 0) |
            (CHAIN_IMPL_FUSED_COMBINE if fused_combine else 0))
    if bits:
        c.implementation_id = bits
    return _ctx(c, workspace)


class PreparedExpertWeights:
    """Expert weights W [E, K, N] laid out once for the grouped GEMM
    (rr_prepare_expert_weights): K-major hi = W and lo = W - trunc_tf32(W)
    in one device buffer twice the size of W. Pass it wherever a chain or
    grouped_gemm_prepared takes expert weights; W itself is not kept."""

    def __init__(self, expert_weights: torch.Tensor, ctx: Context | None = None):
        _need(expert_weights, torch.float32, "expert_weights")
        e, k, n = expert_weights.shape
        self.shape = (e, k, n)
        size = int(lib().rr_prepared_expert_weights_size(e, k, n))
        if size == 0:
            raise ValueError("expert weights must be non-empty")
        self.buffer = torch.empty(size, dtype=torch.uint8, device=expert_weights.device)
        check(lib().rr_prepare_expert_weights(_ptr(expert_weights), e, k, n, _ptr(self.buffer),
                                              size, _ctx(ctx)), "prepare_expert_weights")


def _weights(expert_weights) -> tuple[int | None, tuple[int, int, int], bool]:
    """(pointer, (E, K, N), prepared) of raw or prepared expert weights."""
    if isinstance(expert_weights, PreparedExpertWeights):
        return _ptr(expert_weights.buffer), expert_weights.shape, True
    return _ptr(expert_weights), tuple(expert_weights.shape), False


def _need(t: torch.Tensor | None, dtype: torch.dtype, name: str) -> None:
    if t is None:
        return
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def dense_gemm(a: torch.Tensor, b: torch.Tensor, c: torch.Tensor, m: int, n: int, k: int,
               ctx: Context | None = None) -> None:
    """C[m,n] = A[m,k] . B[k,n] (src/dense_gemm/operator.cpp:18-58)."""
    for t, nm in ((a, "a"), (b, "b"), (c, "c")):
        _need(t, torch.float32, nm)
    check(lib().rr_dense_gemm(_ptr(a), _ptr(b), _ptr(c), m, n, k, _ctx(ctx)), "dense_gemm")


def topk_gate(logits: torch.Tensor, expert_ids: torch.Tensor, weights: torch.Tensor, tokens: int,
              experts: int, top_k: int = 2, ctx: Context | None = None) -> None:
    """Deterministic top-2 selected softmax (src/topk_gate/operator.cpp:18-60)."""
    _need(logits, torch.float32, "logits")
    _need(expert_ids, torch.int32, "expert_ids")
    _need(weights, torch.float32, "weights")
    check(lib().rr_topk_gate(_ptr(logits), _ptr(expert_ids), _ptr(weights), tokens, experts,
                             top_k, _ctx(ctx)), "topk_gate")


def topk_gate_biased(logits: torch.Tensor, logit_bias: torch.Tensor | None,
                     expert_ids: torch.Tensor, weights: torch.Tensor, tokens: int, experts: int,
                     top_k: int = 2, ctx: Context | None = None) -> None:
    """topk_gate over logits + bias[E] (extension; no reference counterpart)."""
    _need(logits, torch.float32, "logits")
    _need(logit_bias, torch.float32, "logit_bias")
    _need(expert_ids, torch.int32, "expert_ids")
    _need(weights, torch.float32, "weights")
    check(lib().rr_topk_gate_biased(_ptr(logits), _ptr(logit_bias), _ptr(expert_ids),
                                    _ptr(weights), tokens, experts, top_k, _ctx(ctx)),
          "topk_gate_biased")


def histogram(expert_ids: torch.Tensor | None, counts: torch.Tensor, route_pairs: int,
              experts: int, ctx: Context | None = None) -> None:
    """counts[e] = #{r : ids[r] == e}, reset included (src/histogram/operator.cpp:20-57)."""
    _need(expert_ids, torch.int32, "expert_ids")
    _need(counts, torch.int32, "counts")
    check(lib().rr_histogram(_ptr(expert_ids), _ptr(counts), route_pairs, experts, _ctx(ctx)),
          "histogram")


def exclusive_scan(counts: torch.Tensor, offsets: torch.Tensor, experts: int,
                   ctx: Context | None = None) -> None:
    """offsets[E+1] from counts[E]; may alias (src/scan/operator.cpp:51-74)."""
    _need(counts, torch.int32, "counts")
    _need(offsets, torch.int32, "offsets")
    check(lib().rr_exclusive_scan(_ptr(counts), _ptr(offsets), experts, _ctx(ctx)),
          "exclusive_scan")


def histogram_exclusive_scan(expert_ids: torch.Tensor | None, counts: torch.Tensor,
                             offsets: torch.Tensor, route_pairs: int, experts: int,
                             ctx: Context | None = None) -> None:
    """Fused histogram + scan (src/scan/operator.cpp:84-134)."""
    _need(expert_ids, torch.int32, "expert_ids")
    _need(counts, torch.int32, "counts")
    _need(offsets, torch.int32, "offsets")
    check(lib().rr_histogram_exclusive_scan(_ptr(expert_ids), _ptr(counts), _ptr(offsets),
                                            route_pairs, experts, _ctx(ctx)),
          "histogram_exclusive_scan")


def token_permute_workspace_size(tokens: int, experts: int, top_k: int, hidden: int = 0) -> int:
    return int(lib().rr_token_permute_workspace_size(tokens, experts, top_k, hidden))


def token_permute(x: torch.Tensor | None, expert_ids: torch.Tensor, offsets: torch.Tensor,
                  x_permuted: torch.Tensor | None, route_pos: torch.Tensor,
                  sorted_route: torch.Tensor | None, tokens: int, experts: int, top_k: int,
                  hidden: int, workspace: torch.Tensor | None,
                  ctx: Context | None = None) -> None:
    """Stable permute (src/permute/operator.cpp:22-83); workspace from
    token_permute_workspace_size (its first E int32 end as the counts)."""
    _need(x, torch.float32, "x")
    _need(x_permuted, torch.float32, "x_permuted")
    for t, nm in ((expert_ids, "expert_ids"), (offsets, "offsets"), (route_pos, "route_pos"),
                  (sorted_route, "sorted_route")):
        _need(t, torch.int32, nm)
    check(lib().rr_token_permute(_ptr(x), _ptr(expert_ids), _ptr(offsets), _ptr(x_permuted),
                                 _ptr(route_pos), _ptr(sorted_route), tokens, experts, top_k,
                                 hidden, _ctx(ctx, workspace)), "token_permute")


def grouped_gemm(x_permuted: torch.Tensor | None, expert_weights: torch.Tensor | None,
                 offsets: torch.Tensor, y_permuted: torch.Tensor, experts: int, hidden: int,
                 output: int, max_expert_tokens: int, ctx: Context | None = None) -> None:
    """Ragged per-expert GEMM (src/grouped_gemm/operator.cpp:17-49)."""
    _need(x_permuted, torch.float32, "x_permuted")
    _need(expert_weights, torch.float32, "expert_weights")
    _need(offsets, torch.int32, "offsets")
    _need(y_permuted, torch.float32, "y_permuted")
    check(lib().rr_grouped_gemm(_ptr(x_permuted), _ptr(expert_weights), _ptr(offsets),
                                _ptr(y_permuted), experts, hidden, output, max_expert_tokens,
                                _ctx(ctx)), "grouped_gemm")


def grouped_gemm_gather(x: torch.Tensor, sorted_route: torch.Tensor, top_k: int,
                        expert_weights: torch.Tensor, offsets: torch.Tensor,
                        y_permuted: torch.Tensor, route_pairs: int,
                        ctx: Context | None = None) -> torch.Tensor:
    """Grouped GEMM whose row r is x[sorted_route[r] // top_k]
    (launch_grouped_gemm_sm86_fp32_gather_v1 of the reference)."""
    experts, hidden, output = expert_weights.shape
    check(lib().rr_grouped_gemm_gather(_ptr(x), _ptr(sorted_route), top_k, _ptr(expert_weights),
                                       _ptr(offsets), _ptr(y_permuted), route_pairs, hidden,
                                       experts, output, _ctx(ctx)), "grouped_gemm_gather")
    return y_permuted


def grouped_gemm_combine(x_permuted: torch.Tensor, expert_weights: torch.Tensor,
                         offsets: torch.Tensor, sorted_route: torch.Tensor,
                         route_weights: torch.Tensor, y: torch.Tensor, route_pairs: int,
                         top_k: int, ctx: Context | None = None) -> torch.Tensor:
    """Grouped GEMM with the unpermute fused into its epilogue
    (rr_grouped_gemm_combine): y [T, N] = sum over each token's routes of
    weight * (x_permuted row . W[e]); top_k 1 or 2."""
    experts, hidden, output = expert_weights.shape
    check(lib().rr_grouped_gemm_combine(_ptr(x_permuted), _ptr(expert_weights), _ptr(offsets),
                                        _ptr(sorted_route), _ptr(route_weights), _ptr(y),
                                        experts, hidden, output, route_pairs, y.shape[0], top_k,
                                        _ctx(ctx)), "grouped_gemm_combine")
    return y


def grouped_gemm_scatter(x_permuted: torch.Tensor, expert_weights: torch.Tensor,
                         offsets: torch.Tensor, row_address: torch.Tensor,
                         bases: torch.Tensor, row_limit: int, route_pairs: int,
                         ctx: Context | None = None) -> None:
    """Grouped GEMM storing output row r at bases[a >> 40] + (a & (2**40 - 1)) * N,
    a = row_address[r] (rr_grouped_gemm_scatter); bases is an int64 device
    tensor of row-buffer pointers."""
    experts, hidden, output = expert_weights.shape
    _need(row_address, torch.int64, "row_address")
    _need(bases, torch.int64, "bases")
    check(lib().rr_grouped_gemm_scatter(_ptr(x_permuted), _ptr(expert_weights), _ptr(offsets),
                                        _ptr(row_address), _ptr(bases), bases.numel(),
                                        row_limit, experts, hidden, output, route_pairs,
                                        _ctx(ctx)), "grouped_gemm_scatter")


def grouped_gemm_prepared(x_permuted: torch.Tensor, weights: PreparedExpertWeights,
                          offsets: torch.Tensor, y_permuted: torch.Tensor, route_pairs: int,
                          ctx: Context | None = None) -> torch.Tensor:
    """Grouped GEMM on prepared expert weights (rr_grouped_gemm_prepared)."""
    _need(x_permuted, torch.float32, "x_permuted")
    _need(offsets, torch.int32, "offsets")
    _need(y_permuted, torch.float32, "y_permuted")
    experts, hidden, output = weights.shape
    check(lib().rr_grouped_gemm_prepared(_ptr(x_permuted), _ptr(weights.buffer), _ptr(offsets),
                                         _ptr(y_permuted), experts, hidden, output, route_pairs,
                                         _ctx(ctx)), "grouped_gemm_prepared")
    return y_permuted


def unpermute(y_permuted: torch.Tensor, route_pos: torch.Tensor, route_weights: torch.Tensor,
              y: torch.Tensor, tokens: int, top_k: int, output: int,
              ctx: Context | None = None) -> None:
    """Weighted combine (src/unpermute/operator.cpp:19-57)."""
    _need(y_permuted, torch.float32, "y_permuted")
    _need(route_pos, torch.int32, "route_pos")
    _need(route_weights, torch.float32, "route_weights")
    _need(y, torch.float32, "y")
    check(lib().rr_unpermute(_ptr(y_permuted), _ptr(route_pos), _ptr(route_weights), _ptr(y),
                             tokens, top_k, output, _ctx(ctx)), "unpermute")


@dataclasses.dataclass
class ChainBuffers:
    """Caller-owned intermediate/output buffers of the L3 chain."""
    logits: torch.Tensor | None
    expert_ids: torch.Tensor
    route_weights: torch.Tensor
    counts: torch.Tensor
    offsets: torch.Tensor
    x_permuted: torch.Tensor
    route_pos: torch.Tensor
    y_permuted: torch.Tensor
    y: torch.Tensor
    workspace: torch.Tensor

    @staticmethod
    def allocate(tokens: int, hidden: int, experts: int, output: int,
                 device: torch.device | str = "cuda", with_logits: bool = True,
                 router_experts: int | None = None) -> "ChainBuffers":
        """`experts` sizes the routing metadata; logits are [tokens,
        router_experts] (default: experts; differs for replicated EP)."""
        f32, i32 = torch.float32, torch.int32
        ws = max(1, chain_workspace_size(tokens, hidden, experts, output))
        re = experts if router_experts is None else router_experts
        return ChainBuffers(
            logits=torch.empty(tokens, re, dtype=f32, device=device) if with_logits else None,
            expert_ids=torch.empty(tokens, 2, dtype=i32, device=device),
            route_weights=torch.empty(tokens, 2, dtype=f32, device=device),
            counts=torch.empty(experts, dtype=i32, device=device),
            offsets=torch.empty(experts + 1, dtype=i32, device=device),
            x_permuted=torch.empty(2 * tokens, hidden, dtype=f32, device=device),
            route_pos=torch.empty(2 * tokens, dtype=i32, device=device),
            y_permuted=torch.empty(2 * tokens, output, dtype=f32, device=device),
            y=torch.empty(tokens, output, dtype=f32, device=device),
            workspace=torch.empty((ws + 255) // 256 * 256, dtype=torch.uint8, device=device),
        )


def chain_workspace_size(tokens: int, hidden: int, experts: int, output: int) -> int:
    return int(lib().rr_chain_workspace_size(tokens, hidden, experts, output))


def chain_from_tokens(x: torch.Tensor, router_weights: torch.Tensor,
                      expert_weights, buf: ChainBuffers,
                      logit_bias: torch.Tensor | None = None,
                      ctx: Context | None = None, gather_rows: bool = False,
                      fused_combine: bool = False) -> torch.Tensor:
    """Seven-stage chain X -> Y (benchmarks/adapters/chain_adapter.cpp:263-467).
    expert_weights: W [E, K, N] or a PreparedExpertWeights.
    gather_rows: the grouped GEMM reads its rows from X (buf.x_permuted is
    not written); fused_combine: the unpermute runs in the grouped GEMM's
    epilogue (buf.y_permuted is not written). Results are bit-identical."""
    tokens, hidden = x.shape
    experts = router_weights.shape[1]
    w_ptr, (_, _, output), prepared = _weights(expert_weights)
    check(lib().rr_chain_from_tokens(
        _ptr(x), _ptr(router_weights), _ptr(logit_bias), w_ptr, _ptr(buf.logits),
        _ptr(buf.expert_ids), _ptr(buf.route_weights), _ptr(buf.counts), _ptr(buf.offsets),
        _ptr(buf.x_permuted), _ptr(buf.route_pos), _ptr(buf.y_permuted), _ptr(buf.y), tokens,
        hidden, experts, output,
        _chain_ctx(ctx, buf.workspace, gather_rows, prepared, fused_combine)),
        "chain_from_tokens")
    return buf.y


def chain_from_logits(logits: torch.Tensor, x: torch.Tensor, expert_weights,
                      buf: ChainBuffers, ctx: Context | None = None,
                      gather_rows: bool = False, fused_combine: bool = False) -> torch.Tensor:
    """Six-stage chain logits -> Y; options as in chain_from_tokens."""
    tokens, hidden = x.shape
    experts = logits.shape[1]
    w_ptr, (_, _, output), prepared = _weights(expert_weights)
    check(lib().rr_chain_from_logits(
        _ptr(logits), _ptr(x), w_ptr, _ptr(buf.expert_ids),
        _ptr(buf.route_weights), _ptr(buf.counts), _ptr(buf.offsets), _ptr(buf.x_permuted),
        _ptr(buf.route_pos), _ptr(buf.y_permuted), _ptr(buf.y), tokens, hidden, experts, output,
        _chain_ctx(ctx, buf.workspace, gather_rows, prepared, fused_combine)),
        "chain_from_logits")
    return buf.y


@dataclasses.dataclass
class RouteChainBuffers:
    """Caller-owned buffers of chain_from_route_ids (R = T * top_k routes)."""
    counts: torch.Tensor
    offsets: torch.Tensor
    x_permuted: torch.Tensor
    route_pos: torch.Tensor
    sorted_route: torch.Tensor | None
    y_permuted: torch.Tensor
    y: torch.Tensor
    workspace: torch.Tensor

    @staticmethod
    def allocate(tokens: int, top_k: int, hidden: int, experts: int, output: int,
                 device: torch.device | str = "cuda",
                 with_sorted_route: bool = True) -> "RouteChainBuffers":
        f32, i32 = torch.float32, torch.int32
        r = tokens * top_k
        ws = max(1, int(lib().rr_route_chain_workspace_size(tokens, top_k, experts)))
        return RouteChainBuffers(
            counts=torch.empty(experts, dtype=i32, device=device),
            offsets=torch.empty(experts + 1, dtype=i32, device=device),
            x_permuted=torch.empty(r, hidden, dtype=f32, device=device),
            route_pos=torch.empty(r, dtype=i32, device=device),
            sorted_route=torch.empty(r, dtype=i32, device=device) if with_sorted_route else None,
            y_permuted=torch.empty(r, output, dtype=f32, device=device),
            y=torch.empty(tokens, output, dtype=f32, device=device),
            workspace=torch.empty((ws + 255) // 256 * 256, dtype=torch.uint8, device=device),
        )


def chain_from_route_ids(x: torch.Tensor, expert_ids: torch.Tensor,
                         route_weights: torch.Tensor, expert_weights: torch.Tensor,
                         buf: RouteChainBuffers, ctx: Context | None = None,
                         gather_rows: bool = False, fused_combine: bool = False) -> torch.Tensor:
    """Post-route chain (benchmarks/adapters/postroute_chain_adapter.cpp:240-354):
    expert_ids / route_weights [T, top_k] -> Y [T, N]. fused_combine needs
    top_k <= 2 and buf.sorted_route."""
    tokens, hidden = x.shape
    top_k = expert_ids.shape[1]
    experts, _, output = expert_weights.shape
    check(lib().rr_chain_from_route_ids(
        _ptr(x), _ptr(expert_ids), _ptr(route_weights), _ptr(expert_weights), _ptr(buf.counts),
        _ptr(buf.offsets), _ptr(buf.x_permuted), _ptr(buf.route_pos), _ptr(buf.sorted_route),
        _ptr(buf.y_permuted), _ptr(buf.y), tokens, top_k, hidden, experts, output,
        _chain_ctx(ctx, buf.workspace, gather_rows, fused_combine=fused_combine)),
        "chain_from_route_ids")
    return buf.y


class Graph:
    """A captured sequence of operator calls (rr_graph_*), replayed with one
    launch. Usage::

        g = Graph.capture(lambda ctx: chain_from_tokens(x, wr, we, buf, ctx=ctx), stream)
        x.copy_(next_tokens); g.launch(stream)

    `stream` is a torch.cuda.Stream (not the default stream); the callable
    receives the Context to pass to every call it makes."""

    def __init__(self, handle: ctypes.c_void_p):
        self._h = handle

    @staticmethod
    def capture(fn, stream: torch.cuda.Stream) -> "Graph":
        ctx = Context(stream=stream.cuda_stream)
        check(lib().rr_graph_capture_begin(ctypes.c_void_p(stream.cuda_stream)),
              "rr_graph_capture_begin")
        try:
            fn(ctx)
        finally:
            h = ctypes.c_void_p()
            st = lib().rr_graph_capture_end(ctypes.c_void_p(stream.cuda_stream), ctypes.byref(h))
        check(st, "rr_graph_capture_end")
        return Graph(h)

    @property
    def nodes(self) -> int:
        return int(lib().rr_graph_node_count(self._h))

    def launch(self, stream: torch.cuda.Stream) -> None:
        check(lib().rr_graph_launch(self._h, ctypes.c_void_p(stream.cuda_stream)),
              "rr_graph_launch")

    def close(self) -> None:
        if self._h:
            lib().rr_graph_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass


class HostChain:
    """chain_from_tokens over host memory (rr_chain_from_tokens_host): chunks
    of `chunk_tokens` stream host -> device, through the chain and back on
    separate copy streams, overlapping the copies with the chain. Y is
    bit-identical to chain_from_tokens over the whole batch.

    input_ready=True (RR_HOST_CHAIN_INPUT_READY): x_host is complete when a
    call is made, so its copies do not wait for earlier work on ctx.stream
    and back-to-back calls overlap."""

    def __init__(self, chunk_tokens: int, hidden: int, experts: int, output: int,
                 input_ready: bool = False):
        self.chunk_tokens, self.hidden, self.experts, self.output = (chunk_tokens, hidden,
                                                                     experts, output)
        h = ctypes.c_void_p()
        check(lib().rr_host_chain_create(chunk_tokens, hidden, experts, output, ctypes.byref(h)),
              "rr_host_chain_create")
        self._h = h
        if input_ready:
            check(lib().rr_host_chain_set_flags(h, 1), "rr_host_chain_set_flags")

    def __call__(self, x_host: torch.Tensor, router_weights: torch.Tensor,
                 expert_weights: torch.Tensor, y_host: torch.Tensor,
                 logit_bias: torch.Tensor | None = None,
                 expert_ids_host: torch.Tensor | None = None,
                 route_weights_host: torch.Tensor | None = None,
                 ctx: Context | None = None) -> torch.Tensor:
        """x_host [T, K] / y_host [T, N] float32 host tensors (pin them for
        overlap); weights on the device. Enqueues; completion is ordered on
        ctx.stream (the default stream when ctx is None)."""
        for t, name in ((x_host, "x_host"), (y_host, "y_host")):
            if t.device.type != "cpu" or t.dtype != torch.float32 or not t.is_contiguous():
                raise ValueError(f"{name} must be a contiguous float32 host tensor")
        tokens = x_host.shape[0]
        check(lib().rr_chain_from_tokens_host(
            self._h, _ptr(x_host), _ptr(router_weights), _ptr(logit_bias),
            _ptr(expert_weights), _ptr(y_host), _ptr(expert_ids_host), _ptr(route_weights_host),
            tokens, _ctx(ctx)), "rr_chain_from_tokens_host")
        return y_host

    def close(self) -> None:
        if self._h:
            lib().rr_host_chain_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass


def kernel_launch_count() -> int:
    return int(lib().rr_kernel_launch_count())


def grouped_gemm_engine(x_permuted: torch.Tensor, expert_weights: torch.Tensor,
                        y_permuted: torch.Tensor, hidden: int, output: int) -> str:
    e = lib().rr_grouped_gemm_engine(_ptr(x_permuted), _ptr(expert_weights), _ptr(y_permuted),
                                     hidden, output)
    return {1: "tcgen05_3xtf32", 2: "fp32_simt", 3: "tcgen05_mixed"}[e]
