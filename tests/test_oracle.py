"""Pins the CPU oracle (CPU only).

The C restatement (oracle/rr_oracle.c) must reproduce the reference's own
known-answer tests and agree with the reference's CPU functions compiled from
its sources (oracle/_ref/librr_ref.so) on seeded inputs, and the committed
golden fixtures (tests/golden/, generated from the reference functions by
tests/golden/make_golden.py).
"""
from __future__ import annotations

import math
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
NAN = float("nan")
INF = float("inf")


# ---- known-answer tests from the reference's own test suite -------------------

def test_top2_kat_operator_api(oracle):
    # tests/operator_api_tests.cpp:626-660
    logits = np.array([[1, 3, 3, 2], [NAN] * 4, [INF, INF, -INF, 0]], np.float32)
    ids, w = oracle.top2_f32(logits)
    assert ids.reshape(-1).tolist() == [1, 2, 0, 1, 0, 1]
    assert w.reshape(-1).tolist() == [0.5] * 6


def test_top2_kat_framework(oracle):
    # tests/correctness_framework_tests.cpp:167-178
    ids, w = oracle.top2_f64(np.array([[NAN, NAN, NAN]]))
    assert ids.reshape(-1).tolist() == [0, 1] and w.reshape(-1).tolist() == [0.5, 0.5]
    ids, w = oracle.top2_f64(np.array([[INF, 2.0, -1.0]]))
    assert w.reshape(-1).tolist() == [1.0, 0.0]


def test_dense_kat(oracle):
    # tests/correctness_tests.cpp:315-318, correctness_framework_tests.cpp:161-163
    c = oracle.dense_gemm_f64(np.array([[1, 2], [3, 4]]), np.array([[5, 6], [7, 8]]))
    assert c.reshape(-1).tolist() == [19.0, 22.0, 43.0, 50.0]


def test_histogram_scan_kat(oracle):
    # tests/operator_api_tests.cpp:662-704 and 706-731
    assert oracle.histogram([0, 1, 1, 1], 2).tolist() == [1, 3]
    assert oracle.histogram(np.zeros(0, np.int32), 2).tolist() == [0, 0]
    for r in (8192, 32768):
        ids = (np.arange(r) & 1).astype(np.int32)
        assert oracle.histogram(ids, 2).tolist() == [r // 2, r // 2]
    assert oracle.exclusive_scan([1, 3]).tolist() == [0, 1, 4]


def test_permute_kat(oracle):
    # tests/correctness_framework_tests.cpp:186-199 (ids {0,1,0,1}, route_pos
    # {0,2,1,3}); tests/operator_api_tests.cpp:734-804 (cursor post-state {2,2}).
    x = np.array([[1, 2], [3, 4]], np.float32)
    ids = np.array([0, 1, 0, 1], np.int32)
    xp, pos, sr, cur = oracle.stable_permute(x, ids, [0, 2, 4], experts=2)
    assert pos.tolist() == [0, 2, 1, 3]
    assert sr.tolist() == [0, 2, 1, 3]
    assert cur.tolist() == [2, 2]
    assert xp.reshape(-1).tolist() == [1, 2, 3, 4, 1, 2, 3, 4]


def test_zero_k_gemm_is_zero(oracle):
    # tests/correctness_framework_tests.cpp:258-275
    y = oracle.grouped_gemm_f64(np.zeros((2, 0), np.float32), np.zeros((1, 0, 2), np.float32),
                                [0, 2])
    assert y.tolist() == [[0.0, 0.0], [0.0, 0.0]]


def test_out_of_range_ids_rejected(oracle):
    with pytest.raises(oracle.OracleError):
        oracle.histogram([0, 5], 2)


# ---- restatement vs the reference's compiled CPU functions ---------------------

needs_ref = pytest.mark.skipif(
    not os.path.exists(os.path.join(os.path.dirname(os.path.dirname(__file__)), "oracle", "_ref",
                                    "librr_ref.so")),
    reason="oracle/_ref not built (needs the reference checkout in the build container)")


def _ref_top2_f32(ref, logits):
    t, e = logits.shape
    ids = np.empty(2 * t, np.int32)
    w = np.empty(2 * t, np.float32)
    rc = ref.rr_ref_top2_f32(logits.ctypes.data_as(__import__("ctypes").POINTER(
        __import__("ctypes").c_float)), t, e, ids.ctypes.data_as(__import__("ctypes").POINTER(
            __import__("ctypes").c_int32)), w.ctypes.data_as(__import__("ctypes").POINTER(
                __import__("ctypes").c_float)))
    assert rc == 0
    return ids.reshape(t, 2), w.reshape(t, 2)


@needs_ref
@pytest.mark.parametrize("experts", [2, 3, 8, 63, 64, 128, 256])
def test_top2_port_matches_reference(oracle, experts):
    import ctypes
    rng = np.random.default_rng(experts)
    t = 257
    logits = rng.standard_normal((t, experts)).astype(np.float32)
    logits[::7, 0] = logits[::7, -1]            # ties
    logits[::11] = np.round(logits[::11])       # many ties
    logits[::13, 1] = np.nan
    logits[5] = np.nan                          # all-NaN row
    logits[6, 0] = np.inf
    logits[9, :] = -np.inf
    logits[10, 1] = -0.0
    logits[10, 0] = 0.0
    ids_p, w_p = oracle.top2_f32(logits)
    ids_r, w_r = _ref_top2_f32(oracle.ref, logits)
    assert np.array_equal(ids_p, ids_r)
    assert np.array_equal(w_p, w_r)
    # double-precision variant
    l64 = logits.astype(np.float64)
    ids_d = np.empty(2 * t, np.int32)
    w_d = np.empty(2 * t, np.float64)
    assert oracle.ref.rr_ref_top2_f64(l64.ctypes.data_as(ctypes.POINTER(ctypes.c_double)), t,
                                      experts, ids_d.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                                      w_d.ctypes.data_as(ctypes.POINTER(ctypes.c_double))) == 0
    ids_pd, w_pd = oracle.top2_f64(l64)
    assert np.array_equal(ids_pd.reshape(-1), ids_d)
    assert np.array_equal(w_pd.reshape(-1), w_d)


@needs_ref
@pytest.mark.parametrize("experts,dist", [(1, "uniform"), (8, "zipf"), (64, "uniform"),
                                          (256, "one"), (1024, "uniform")])
def test_histogram_scan_port_matches_reference(oracle, experts, dist):
    import ctypes
    from raggedroute_b200.workloads import route_ids
    ids = route_ids(100_003, experts, dist, seed=experts)
    c_ref = np.empty(experts, np.int32)
    assert oracle.ref.rr_ref_histogram(ids.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                                       ids.size, experts,
                                       c_ref.ctypes.data_as(ctypes.POINTER(ctypes.c_int32))) == 0
    c = oracle.histogram(ids, experts)
    assert np.array_equal(c, c_ref)
    o_ref = np.empty(experts + 1, np.int32)
    assert oracle.ref.rr_ref_exclusive_scan(c.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                                            experts,
                                            o_ref.ctypes.data_as(ctypes.POINTER(ctypes.c_int32))) == 0
    assert np.array_equal(oracle.exclusive_scan(c), o_ref)


@needs_ref
@pytest.mark.parametrize("tokens,experts,top_k,hidden", [(2, 2, 2, 2), (33, 7, 3, 5),
                                                         (500, 64, 2, 16), (129, 256, 1, 3)])
def test_stable_permute_passes_reference_validator(oracle, tokens, experts, top_k, hidden):
    import ctypes
    rng = np.random.default_rng(tokens)
    x = rng.uniform(-1, 1, (tokens, hidden)).astype(np.float32)
    ids = rng.integers(0, experts, tokens * top_k).astype(np.int32)
    offsets = oracle.exclusive_scan(oracle.histogram(ids, experts))
    xp, pos, sr, cur = oracle.stable_permute(x, ids, offsets, experts, top_k)
    f = ctypes.POINTER(ctypes.c_float)
    i = ctypes.POINTER(ctypes.c_int32)
    ok = oracle.ref.rr_ref_validate_permute(x.ctypes.data_as(f), ids.ctypes.data_as(i),
                                            offsets.ctypes.data_as(i), experts,
                                            xp.ctypes.data_as(f), pos.ctypes.data_as(i),
                                            sr.ctypes.data_as(i), tokens, top_k, hidden)
    assert ok == 1
    assert np.array_equal(cur, oracle.histogram(ids, experts))
    assert np.array_equal(pos, oracle.stable_route_pos(ids, offsets, experts))


@needs_ref
def test_contractions_port_match_reference(oracle):
    import ctypes
    rng = np.random.default_rng(7)
    f = ctypes.POINTER(ctypes.c_float)
    d = ctypes.POINTER(ctypes.c_double)
    i = ctypes.POINTER(ctypes.c_int32)
    a = rng.uniform(-1, 1, (37, 29)).astype(np.float32)
    b = rng.uniform(-1, 1, (29, 11)).astype(np.float32)
    c_ref = np.empty((37, 11))
    assert oracle.ref.rr_ref_dense_gemm(a.ctypes.data_as(f), b.ctypes.data_as(f),
                                        c_ref.ctypes.data_as(d), 37, 11, 29) == 0
    assert np.array_equal(oracle.dense_gemm_f64(a, b), c_ref)
    sizes = np.array([5, 0, 17, 3], np.int32)
    offsets = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int32)
    x = rng.uniform(-1, 1, (25, 13)).astype(np.float32)
    w = rng.normal(0, 0.3, (4, 13, 9)).astype(np.float32)
    y_ref = np.empty((25, 9))
    assert oracle.ref.rr_ref_grouped_gemm(x.ctypes.data_as(f), w.ctypes.data_as(f),
                                          offsets.ctypes.data_as(i), 4, 13, 9,
                                          y_ref.ctypes.data_as(d)) == 0
    y = oracle.grouped_gemm_f64(x, w, offsets)
    np.testing.assert_allclose(y, y_ref, rtol=1e-13, atol=1e-13)
    pos = rng.permutation(24).astype(np.int32)
    yp = rng.uniform(-1, 1, (24, 9)).astype(np.float32)
    rw = rng.uniform(0, 1, 24).astype(np.float32)
    u_ref = np.empty((12, 9))
    assert oracle.ref.rr_ref_unpermute(yp.ctypes.data_as(f), pos.ctypes.data_as(i),
                                       rw.ctypes.data_as(f), 12, 2, 9,
                                       u_ref.ctypes.data_as(d)) == 0
    np.testing.assert_allclose(oracle.unpermute_f64(yp, pos, rw), u_ref, rtol=1e-15, atol=1e-15)


@needs_ref
def test_reference_cpu_chain_runs(oracle):
    """The threaded reference chain used by bench.py --impl reference agrees
    with the port's float chain within the reference's chain tolerance."""
    import ctypes
    rng = np.random.default_rng(11)
    t, k, e, n = 64, 32, 8, 16
    x = rng.uniform(-1, 1, (t, k)).astype(np.float32)
    wr = rng.normal(0, 1 / math.sqrt(k), (k, e)).astype(np.float32)
    we = rng.normal(0, 1 / math.sqrt(k), (e, k, n)).astype(np.float32)
    y = np.empty((t, n), np.float32)
    f = ctypes.POINTER(ctypes.c_float)
    assert oracle.ref.rr_ref_chain_from_tokens(x.ctypes.data_as(f), wr.ctypes.data_as(f), None,
                                               we.ctypes.data_as(f), t, k, e, n, 4,
                                               y.ctypes.data_as(f)) == 0
    logits = oracle.chain_logits_f32(x, wr)
    ids, w = oracle.top2_f32(logits)
    y_port = oracle.chain_output_f32(x, we, ids, w)
    ok, _, _ = oracle.compare_floating(y, y_port, 1e-4, 4e-5 * k)
    assert ok


# ---- committed golden fixtures -------------------------------------------------

def _golden(name):
    path = os.path.join(GOLDEN, name)
    assert os.path.exists(path), f"missing golden fixture {path}; run tests/golden/make_golden.py"
    return np.load(path)


def test_golden_topk(oracle):
    g = _golden("topk_c2_slice.npz")
    ids, w = oracle.top2_f32(g["logits"])
    assert np.array_equal(ids, g["ids"])
    np.testing.assert_allclose(w, g["weights"], rtol=1e-6, atol=1e-6)


def test_golden_chain_c1(oracle):
    g = _golden("chain_c1_small.npz")
    logits = oracle.chain_logits_f32(g["x"], g["router_w"])
    ids, w = oracle.top2_f32(logits)
    np.testing.assert_allclose(w, g["weights"], rtol=1e-6, atol=1e-6)
    assert np.array_equal(ids, g["ids"])
    counts = oracle.histogram(ids, g["router_w"].shape[1])
    assert np.array_equal(counts, g["counts"])
    assert np.array_equal(oracle.exclusive_scan(counts), g["offsets"])
    y = oracle.chain_output_f32(g["x"], g["expert_w"], ids, w)
    ok, _, _ = oracle.compare_floating(y, g["y_ref_f64"], 1e-4, 4e-5 * g["x"].shape[1])
    assert ok


def test_golden_permute(oracle):
    g = _golden("permute_small.npz")
    xp, pos, sr, cur = oracle.stable_permute(g["x"], g["ids"], g["offsets"],
                                             experts=g["cursors"].size, top_k=2)
    assert np.array_equal(pos, g["route_pos"])
    assert np.array_equal(sr, g["sorted_route"])
    assert np.array_equal(cur, g["cursors"])


@pytest.mark.parametrize("top_k", [1, 2, 4, 8])
@pytest.mark.parametrize("dist", ["uniform", "zipf", "duplicate_route", "single_hot",
                                  "round_robin"])
def test_route_chain_oracle_matches_reference_formula(oracle, top_k, dist):
    """The post-route chain composed from the stage oracles equals the
    reference's float restatement (postroute_chain_adapter.cpp:654-675)
    within its tolerance (atol 1e-4, rtol 4e-5*K*top_k), and its routing
    metadata is the stable bijection onto expert segments."""
    from route_ids import make_route_ids, make_route_weights
    t, k, e, n = 17, 64, 16, 64
    rng = np.random.default_rng(top_k)
    x = rng.uniform(-1, 1, (t, k)).astype(np.float32)
    w = rng.normal(0, 1 / 8, (e, k, n)).astype(np.float32)
    ids = make_route_ids(t, top_k, e, dist, 1.4, seed=top_k)
    rw = make_route_weights(t, top_k, seed=top_k)
    counts, offsets, xp, pos, sr, y = oracle.route_chain_f64(x, w, ids, rw, e)
    ref = oracle.route_chain_output_f32(x, w, ids, rw)
    ok, _, _ = oracle.compare_floating(y.astype(np.float32), ref, 1e-4, 4e-5 * k * top_k)
    assert ok
    flat = ids.reshape(-1)
    assert np.array_equal(counts, np.bincount(flat, minlength=e))
    for r in range(flat.size):
        assert offsets[flat[r]] <= pos[r] < offsets[flat[r] + 1]
        assert sr[pos[r]] == r
        assert np.array_equal(xp[pos[r]], x[r // top_k])
