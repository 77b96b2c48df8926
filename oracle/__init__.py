"""CPU oracle for the RaggedRoute routing path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its
``cpu_baseline`` leg and ``--impl reference``) may import this package, and
only as the checker or the timed CPU baseline; the product path in
``raggedroute_b200`` never does.

Two independent CPU implementations are exposed:

* ``port``: ``oracle/rr_oracle.c``, this repository's plain-C restatement of
  the reference algorithm (each function cites the reference file:line).
* ``ref``:  ``oracle/_ref/librr_ref.so``, RaggedRoute's own CPU reference
  functions compiled from its sources (``oracle/build_oracle.py``). Present
  wherever the build container produced it; the tests pin ``port`` against it
  and against the reference's known-answer tests.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

_i32p = ctypes.POINTER(ctypes.c_int32)
_f32p = ctypes.POINTER(ctypes.c_float)
_f64p = ctypes.POINTER(ctypes.c_double)
_int = ctypes.c_int
_i64 = ctypes.c_int64


def _p(a: np.ndarray | None, typ):
    if a is None:
        return ctypes.cast(None, typ)
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(typ)


def _load_port() -> ctypes.CDLL:
    path = os.path.join(HERE, "librr_oracle.so")
    if not os.path.exists(path):
        from oracle.build_oracle import build_oracle  # noqa: WPS433
        build_oracle()
    lib = ctypes.CDLL(path)
    sigs = {
        "rr_oracle_top2_f64": [_f64p, _int, _int, _i32p, _f64p],
        "rr_oracle_top2_f32": [_f32p, _f32p, _int, _int, _i32p, _f32p],
        "rr_oracle_histogram": [_i32p, _i64, _int, _i32p],
        "rr_oracle_exclusive_scan": [_i32p, _int, _i32p],
        "rr_oracle_stable_permute": [_f32p, _i32p, _i32p, _int, _int, _int, _int, _f32p, _i32p,
                                     _i32p, _i32p],
        "rr_oracle_dense_gemm_f64": [_f32p, _f32p, _f64p, _int, _int, _int],
        "rr_oracle_grouped_gemm_f64": [_f32p, _f32p, _i32p, _int, _int, _int, _f64p],
        "rr_oracle_unpermute_f64": [_f32p, _i32p, _f32p, _int, _int, _int, _f64p],
        "rr_oracle_chain_logits_f32": [_f32p, _f32p, _int, _int, _int, _f32p],
        "rr_oracle_chain_output_f32": [_f32p, _f32p, _i32p, _f32p, _int, _int, _int, _int, _f32p],
        "rr_oracle_route_chain_output_f32": [_f32p, _f32p, _i32p, _f32p, _int, _int, _int, _int,
                                             _int, _f32p],
    }
    for name, argtypes in sigs.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = _int
    return lib


def _load_ref() -> ctypes.CDLL | None:
    path = os.path.join(HERE, "_ref", "librr_ref.so")
    if not os.path.exists(path):
        return None
    lib = ctypes.CDLL(path)
    sigs = {
        "rr_ref_top2_f64": [_f64p, _int, _int, _i32p, _f64p],
        "rr_ref_top2_f32": [_f32p, _int, _int, _i32p, _f32p],
        "rr_ref_histogram": [_i32p, _i64, _int, _i32p],
        "rr_ref_exclusive_scan": [_i32p, _int, _i32p],
        "rr_ref_validate_permute": [_f32p, _i32p, _i32p, _int, _f32p, _i32p, _i32p, _int, _int,
                                    _int],
        "rr_ref_dense_gemm": [_f32p, _f32p, _f64p, _int, _int, _int],
        "rr_ref_grouped_gemm": [_f32p, _f32p, _i32p, _int, _int, _int, _f64p],
        "rr_ref_unpermute": [_f32p, _i32p, _f32p, _int, _int, _int, _f64p],
        "rr_ref_chain_from_tokens": [_f32p, _f32p, _f32p, _f32p, _int, _int, _int, _int, _int,
                                     _f32p],
    }
    for name, argtypes in sigs.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = _int
    return lib


port = _load_port()
ref = _load_ref()


class OracleError(RuntimeError):
    pass


def _check(rc: int, what: str) -> None:
    if rc != 0:
        raise OracleError(f"{what} rejected its input (code {rc})")


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def _i32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.int32)


# --------------------------------------------------------------------------
# Port (C restatement)
# --------------------------------------------------------------------------

def top2_f32(logits, bias=None):
    """Float top-2 selected softmax (adapter_utils.h:363-418); optional bias[E]."""
    logits = _f32(logits)
    t, e = logits.shape
    ids = np.empty((t, 2), np.int32)
    w = np.empty((t, 2), np.float32)
    b = None if bias is None else _f32(bias)
    _check(port.rr_oracle_top2_f32(_p(logits, _f32p), _p(b, _f32p), t, e, _p(ids, _i32p),
                                   _p(w, _f32p)), "top2_f32")
    return ids, w


def top2_f64(logits):
    """Double top-2 selected softmax (topk_gate/cpu_reference/reference.cpp:12-72)."""
    logits = np.ascontiguousarray(logits, dtype=np.float64)
    t, e = logits.shape
    ids = np.empty((t, 2), np.int32)
    w = np.empty((t, 2), np.float64)
    _check(port.rr_oracle_top2_f64(_p(logits, _f64p), t, e, _p(ids, _i32p), _p(w, _f64p)),
           "top2_f64")
    return ids, w


def histogram(ids, experts: int):
    ids = _i32(ids).reshape(-1)
    counts = np.empty(experts, np.int32)
    _check(port.rr_oracle_histogram(_p(ids, _i32p), ids.size, experts, _p(counts, _i32p)),
           "histogram")
    return counts


def exclusive_scan(counts):
    counts = _i32(counts)
    offsets = np.empty(counts.size + 1, np.int32)
    _check(port.rr_oracle_exclusive_scan(_p(counts, _i32p), counts.size, _p(offsets, _i32p)),
           "exclusive_scan")
    return offsets


def stable_permute(x, ids, offsets, experts: int, top_k: int = 2, with_rows: bool = True):
    """Returns (x_permuted, route_pos, sorted_route, cursors) in the stable order."""
    x = _f32(x)
    ids = _i32(ids).reshape(-1)
    offsets = _i32(offsets)
    tokens, hidden = x.shape
    routes = tokens * top_k
    xp = np.empty((routes, hidden), np.float32) if with_rows else None
    pos = np.empty(routes, np.int32)
    sr = np.empty(routes, np.int32)
    cur = np.empty(experts, np.int32)
    _check(port.rr_oracle_stable_permute(_p(x, _f32p), _p(ids, _i32p), _p(offsets, _i32p),
                                         tokens, top_k, hidden if with_rows else 0, experts,
                                         _p(xp, _f32p), _p(pos, _i32p), _p(sr, _i32p),
                                         _p(cur, _i32p)), "stable_permute")
    return xp, pos, sr, cur


def stable_route_pos(ids, offsets, experts: int):
    """Route positions only (no rows), numpy-vectorised for large R."""
    ids = _i32(ids).reshape(-1)
    order = np.argsort(ids, kind="stable")
    pos = np.empty(ids.size, np.int32)
    pos[order] = np.arange(ids.size, dtype=np.int32)
    # Within each expert the rank is pos - (first index of that expert in the
    # sorted order) which equals offsets[e] when offsets match the histogram.
    counts = np.bincount(ids, minlength=experts).astype(np.int64)
    starts = np.concatenate([[0], np.cumsum(counts)[:-1]])
    pos = (pos - starts[ids] + _i32(offsets)[ids]).astype(np.int32)
    return pos


def dense_gemm_f64(a, b):
    a = _f32(a)
    b = _f32(b)
    m, k = a.shape
    k2, n = b.shape
    assert k == k2
    c = np.empty((m, n), np.float64)
    _check(port.rr_oracle_dense_gemm_f64(_p(a, _f32p), _p(b, _f32p), _p(c, _f64p), m, n, k),
           "dense_gemm")
    return c


def grouped_gemm_f64(x, w, offsets):
    x = _f32(x)
    w = _f32(w)
    offsets = _i32(offsets)
    experts, hidden, output = w.shape
    y = np.zeros((x.shape[0], output), np.float64)
    _check(port.rr_oracle_grouped_gemm_f64(_p(x, _f32p), _p(w, _f32p), _p(offsets, _i32p),
                                           experts, hidden, output, _p(y, _f64p)), "grouped_gemm")
    return y


def unpermute_f64(yp, route_pos, route_weights, top_k: int = 2):
    yp = _f32(yp)
    route_pos = _i32(route_pos).reshape(-1)
    route_weights = _f32(route_weights).reshape(-1)
    routes, output = yp.shape
    tokens = route_pos.size // top_k
    y = np.empty((tokens, output), np.float64)
    _check(port.rr_oracle_unpermute_f64(_p(yp, _f32p), _p(route_pos, _i32p),
                                        _p(route_weights, _f32p), tokens, top_k, output,
                                        _p(y, _f64p)), "unpermute")
    return y


def _ftz(v: np.ndarray) -> np.ndarray:
    """float32 values below 2^-126 in magnitude replaced by a zero of the
    same sign."""
    tiny = np.abs(v) < np.float32(2.0 ** -126)
    return np.where(tiny, np.copysign(np.float32(0.0), v), v).astype(np.float32)


def unpermute_f32_ftz(yp, route_pos, route_weights, top_k: int = 2) -> np.ndarray:
    """The library's unpermute arithmetic in float32, bit for bit: from 0.0f,
    in rank order, acc = ftz(ftz(acc) + ftz(rn(w * v))) -- the rounded
    product added with round-to-nearest and subnormal operands and result
    flushed to zero (what a global float reduction does on the GPU, so the
    grouped GEMM's fused combine gives the same sum). The reference's own
    unpermute (src/unpermute/cuda_naive/baseline.cu:13-30) sums the same
    terms in the same order with fused multiply-adds; unpermute_f64 is its
    exact value."""
    yp = _f32(yp)
    route_pos = _i32(route_pos).reshape(-1)
    w = _f32(route_weights).reshape(-1)
    tokens = route_pos.size // top_k
    acc = np.zeros((tokens, yp.shape[1]), np.float32)
    for k in range(top_k):
        pos = route_pos[k::top_k]
        prod = _ftz((w[k::top_k][:, None] * yp[pos]).astype(np.float32))
        acc = _ftz((_ftz(acc) + prod).astype(np.float32))
    return acc


def chain_logits_f32(x, router_w):
    x = _f32(x)
    router_w = _f32(router_w)
    t, k = x.shape
    e = router_w.shape[1]
    out = np.empty((t, e), np.float32)
    _check(port.rr_oracle_chain_logits_f32(_p(x, _f32p), _p(router_w, _f32p), t, k, e,
                                           _p(out, _f32p)), "chain_logits")
    return out


def chain_output_f32(x, expert_w, ids, weights):
    x = _f32(x)
    expert_w = _f32(expert_w)
    ids = _i32(ids).reshape(-1)
    weights = _f32(weights).reshape(-1)
    t, k = x.shape
    e, _, n = expert_w.shape
    y = np.empty((t, n), np.float32)
    _check(port.rr_oracle_chain_output_f32(_p(x, _f32p), _p(expert_w, _f32p), _p(ids, _i32p),
                                           _p(weights, _f32p), t, k, n, e, _p(y, _f32p)),
           "chain_output")
    return y


def chain_output_f64(x, expert_w, ids, weights):
    """The chain output in double: Y[t] = sum_k w[t,k] * (X[t] . W[ids[t,k]]),
    the same composition as the float chain oracle
    (benchmarks/adapters/chain_adapter.cpp:858-879) without its float
    rounding. Routing (ids, weights) is an input, so a caller checks the
    device's outputs against it with the device's own (exactly checked)
    routing. Returns float64 [T, N]."""
    x = np.asarray(x, np.float64)
    expert_w = np.asarray(expert_w, np.float64)
    ids = _i32(ids)
    ids = ids.reshape(x.shape[0], -1)
    weights = np.asarray(weights, np.float64).reshape(ids.shape)
    y = np.zeros((x.shape[0], expert_w.shape[2]), np.float64)
    for e in np.unique(ids):
        rows, ranks = np.nonzero(ids == e)
        np.add.at(y, rows, weights[rows, ranks][:, None] * (x[rows] @ expert_w[e]))
    return y


def route_chain_output_f32(x, expert_w, ids, weights):
    """Post-route chain output in float, rank order (postroute_chain_adapter.cpp:654-675)."""
    x = _f32(x)
    expert_w = _f32(expert_w)
    ids = _i32(ids)
    top_k = ids.shape[1]
    ids = ids.reshape(-1)
    weights = _f32(weights).reshape(-1)
    t, k = x.shape
    e, _, n = expert_w.shape
    y = np.empty((t, n), np.float32)
    _check(port.rr_oracle_route_chain_output_f32(_p(x, _f32p), _p(expert_w, _f32p),
                                                 _p(ids, _i32p), _p(weights, _f32p), t, top_k,
                                                 k, n, e, _p(y, _f32p)), "route_chain_output")
    return y


def route_chain_f64(x, expert_w, ids, weights, experts: int):
    """Post-route chain composed from the stage oracles (histogram, scan,
    stable permute, grouped GEMM and unpermute in double): returns counts,
    offsets, x_permuted, route_pos, sorted_route and y (float64)."""
    ids = _i32(ids)
    top_k = ids.shape[1]
    counts = histogram(ids.reshape(-1), experts)
    offsets = exclusive_scan(counts)
    xp, pos, sr, _ = stable_permute(x, ids, offsets, experts, top_k)
    yp = grouped_gemm_f64(xp, expert_w, offsets).astype(np.float32)
    y = unpermute_f64(yp, pos, weights, top_k)
    return counts, offsets, xp, pos, sr, y


# --------------------------------------------------------------------------
# Comparators (the reference's tolerance rules)
# --------------------------------------------------------------------------

def gemm_error_bound(a, b, k: int):
    """Accumulation-aware bound 4*gamma_K*sum|a||b| + 1e-7 of
    src/correctness/reference_validation.cpp:70-115 (u = 2^-24 for FP32)."""
    u = 2.0 ** -24
    gamma = k * u / (1.0 - k * u)
    return 4.0 * gamma * (np.abs(np.asarray(a, np.float64)) @ np.abs(np.asarray(b, np.float64))) \
        + 1e-7


def _numeric_class(v: np.ndarray) -> np.ndarray:
    return np.where(np.isnan(v), 2, np.where(np.isinf(v), 1 + 3 * (v > 0), 0))


def compare_floating(actual, expected, atol: float, rtol: float) -> tuple[bool, float, float]:
    """Elementwise |a - e| <= atol + rtol * max(|e|, 1e-30) on finite values,
    with NaN/Inf/finite classes required to match
    (src/correctness/reference_validation.cpp:32-68).
    Returns (ok, max_abs_error, max_rel_error)."""
    a = np.asarray(actual, np.float64).reshape(-1)
    e = np.asarray(expected, np.float64).reshape(-1)
    if a.shape != e.shape:
        return False, float("inf"), float("inf")
    class_ok = _numeric_class(a) == _numeric_class(e)
    finite = np.isfinite(e) & class_ok
    denom = np.maximum(np.abs(e), 1e-30)
    err = np.where(finite, np.abs(a - e), 0.0)
    ok = bool(np.all(class_ok) and np.all(err <= atol + rtol * denom))
    return ok, float(err.max(initial=0.0)), float((err / denom).max(initial=0.0))


def normwise_rel_error(actual, expected) -> float:
    """||a - e||_2 / ||e||_2 over finite entries."""
    a = np.asarray(actual, np.float64).reshape(-1)
    e = np.asarray(expected, np.float64).reshape(-1)
    m = np.isfinite(e)
    den = np.linalg.norm(e[m])
    num = np.linalg.norm(a[m] - e[m])
    return float(num / den) if den > 0 else float(num)
