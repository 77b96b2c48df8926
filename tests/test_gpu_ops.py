"""GPU parity of every operator against the CPU oracle, through the C ABI.

Integer/index outputs (ids, counts, offsets, route_pos, sorted_route,
cursors) and permuted rows must be bit-exact. Floating outputs use the
reference's tolerances: gate weights 1e-6 abs/rel
(benchmarks/adapters/topk_gate_adapter.cpp:157), unpermute (1e-6, 1e-5)
(unpermute_adapter.cpp:134), GEMMs the accumulation-aware bound
4*gamma_K*sum|a||b| + 1e-7 (src/correctness/reference_validation.cpp:70-115)
plus a normwise relative error <= 1e-5 against the FP64 oracle.
"""
from __future__ import annotations

import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

NAN = float("nan")
INF = float("inf")


def dev(a, device, dtype=None):
    t = torch.as_tensor(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    return t.to(device)


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


# ---- topk_gate ------------------------------------------------------------------

def test_topk_kat(rrlib, oracle, cuda):
    # tests/operator_api_tests.cpp:626-660, for every kernel family/id the
    # reference accepts.
    logits = dev(np.array([[1, 3, 3, 2], [NAN] * 4, [INF, INF, -INF, 0]], np.float32), cuda)
    ids = torch.empty(3, 2, dtype=torch.int32, device=cuda)
    w = torch.empty(3, 2, dtype=torch.float32, device=cuda)
    for fam, impl in [(0, 0), (1, 0), (2, 1), (2, 2), (2, 3), (2, 4)]:
        ids.fill_(-7)
        rrlib.topk_gate(logits, ids, w, 3, 4, ctx=rrlib.Context(kernel_family=fam,
                                                                  implementation_id=impl))
        assert host(ids).reshape(-1).tolist() == [1, 2, 0, 1, 0, 1]
        assert host(w).reshape(-1).tolist() == [0.5] * 6


def _topk_check(rrlib, oracle, cuda, logits_np, bias_np=None):
    t, e = logits_np.shape
    ids = torch.empty(t, 2, dtype=torch.int32, device=cuda)
    w = torch.empty(t, 2, dtype=torch.float32, device=cuda)
    rrlib.topk_gate(dev(logits_np, cuda), ids, w, t, e)
    ids_ref, w_ref = oracle.top2_f32(logits_np)
    assert np.array_equal(host(ids), ids_ref)
    ok, err, _ = oracle.compare_floating(host(w), w_ref, 1e-6, 1e-6)
    assert ok, err


@pytest.mark.parametrize("experts", [2, 3, 4, 5, 7, 8, 16, 31, 32, 63, 64, 65, 128, 256, 1000,
                                     1024])
@pytest.mark.parametrize("tokens", [1, 7, 65, 1000])
def test_topk_random_shapes(rrlib, oracle, cuda, experts, tokens):
    rng = np.random.default_rng(experts * 1000 + tokens)
    logits = rng.standard_normal((tokens, experts)).astype(np.float32)
    logits[::3] = np.round(logits[::3] * 2) / 2  # frequent ties
    _topk_check(rrlib, oracle, cuda, logits)


@pytest.mark.parametrize("mode", ["duplicate_max", "ties", "all_nan", "signed_zero",
                                  "mixed_nan_neg_inf", "single_infinity", "multiple_infinity",
                                  "extreme"])
def test_topk_special_modes(rrlib, oracle, cuda, mode):
    # Special-value modes of tests/correctness_tests.cpp:629-640 at T=33, E=63.
    rng = np.random.default_rng(3)
    t, e = 33, 63
    x = rng.standard_normal((t, e)).astype(np.float32)
    if mode == "duplicate_max":
        x[:, 5] = x.max(axis=1) + 1
        x[:, 40] = x[:, 5]
    elif mode == "ties":
        x[:] = 1.0
    elif mode == "all_nan":
        x[:] = NAN
    elif mode == "signed_zero":
        x[:] = -1.0
        x[:, 3] = -0.0
        x[:, 9] = 0.0
    elif mode == "mixed_nan_neg_inf":
        x[:, ::2] = NAN
        x[:, 1::2] = -INF
        x[::5, 7] = 0.5
    elif mode == "single_infinity":
        x[:, 11] = INF
    elif mode == "multiple_infinity":
        x[:, 2] = INF
        x[:, 50] = INF
        x[::2, 60] = -INF
    elif mode == "extreme":
        x[:, 0] = 3.4e38
        x[:, 1] = -3.4e38
        x[::3, 2] = 1e-45
    _topk_check(rrlib, oracle, cuda, x)


@pytest.mark.parametrize("experts", [4, 8, 36, 64, 100, 128, 256, 1024])
@pytest.mark.parametrize("tokens", [16384, 40001])
@pytest.mark.parametrize("biased", [False, True])
def test_topk_large_batches(rrlib, oracle, cuda, experts, tokens, biased):
    """Batches of 16384 rows and more take the streaming instance (8 loads
    per lane in one pass, an L2 bulk prefetch of every row group a CTA
    ranks): rows exactly covered by the lanes' loads (E = 64 .. 1024) and
    rows covered in part (E = 4, 8 with one lane per row; E = 36 and 100
    with 2 and 4 lanes, some of whose load slots lie past the row). Ids
    bit-exact and weights within the reference's 1e-6 against the oracle,
    with ties, NaN rows, infinities and signed zeros spread over the row
    groups and a ragged last group."""
    rng = np.random.default_rng(experts * 7 + tokens + biased)
    x = rng.standard_normal((tokens, experts)).astype(np.float32)
    x[::3] = np.round(x[::3] * 2) / 2
    x[5::97] = NAN
    x[7::89, experts // 2] = INF
    x[11::83, 0] = -INF
    x[13::79, :] = -0.0
    x[17::71, experts - 1] = 0.0
    bias = rng.standard_normal(experts).astype(np.float32) if biased else None
    ids = torch.full((tokens, 2), -9, dtype=torch.int32, device=cuda)
    w = torch.empty(tokens, 2, dtype=torch.float32, device=cuda)
    if biased:
        rrlib.topk_gate_biased(dev(x, cuda), dev(bias, cuda), ids, w, tokens, experts)
    else:
        rrlib.topk_gate(dev(x, cuda), ids, w, tokens, experts)
    ids_ref, w_ref = oracle.top2_f32(x, bias)
    assert np.array_equal(host(ids), ids_ref)
    ok, err, _ = oracle.compare_floating(host(w), w_ref, 1e-6, 1e-6)
    assert ok, err


def test_topk_c2_logits(rrlib, oracle, cuda):
    from raggedroute_b200.workloads import c2_logits
    _topk_check(rrlib, oracle, cuda, c2_logits())


def test_topk_misaligned_rows(rrlib, oracle, cuda):
    # Row stride not a multiple of 16 bytes and a base offset of 4 bytes.
    rng = np.random.default_rng(9)
    t, e = 100, 12
    buf = torch.empty(t * e + 1, dtype=torch.float32, device=cuda)
    logits = rng.standard_normal((t, e)).astype(np.float32)
    buf[1:] = dev(logits.reshape(-1), cuda)
    ids = torch.empty(2 * t + 1, dtype=torch.int32, device=cuda)
    w = torch.empty(2 * t + 1, dtype=torch.float32, device=cuda)
    rrlib.topk_gate(buf[1:], ids[1:], w[1:], t, e)
    ids_ref, w_ref = oracle.top2_f32(logits)
    assert np.array_equal(host(ids[1:]).reshape(t, 2), ids_ref)
    assert oracle.compare_floating(host(w[1:]).reshape(t, 2), w_ref, 1e-6, 1e-6)[0]


def test_topk_rejects_bad_args(rrlib, cuda):
    logits = torch.zeros(2, 4, device=cuda)
    ids = torch.empty(2, 2, dtype=torch.int32, device=cuda)
    w = torch.empty(2, 2, device=cuda)
    for t, e, k in [(2, 1, 2), (2, 1025, 2), (2, 4, 3), (-1, 4, 2)]:
        with pytest.raises(rrlib.RaggedRouteError) as ei:
            rrlib.topk_gate(logits, ids, w, t, e, top_k=k)
        assert ei.value.code == rrlib.StatusCode.INVALID_ARGUMENT


# ---- histogram / scan -------------------------------------------------------------

def test_histogram_reset_kat(rrlib, cuda):
    # tests/operator_api_tests.cpp:662-731
    ids = dev(np.array([0, 1, 1, 1], np.int32), cuda)
    counts = dev(np.array([99, 99], np.int32), cuda)
    rrlib.histogram(ids, counts, 4, 2)
    assert host(counts).tolist() == [1, 3]
    counts.copy_(torch.tensor([77, 88], dtype=torch.int32))
    rrlib.histogram(None, counts, 0, 2)
    assert host(counts).tolist() == [0, 0]
    for r in (8192, 32768):
        ids = dev((np.arange(r) & 1).astype(np.int32), cuda)
        counts = dev(np.array([9, 9], np.int32), cuda)
        rrlib.histogram(ids, counts, r, 2, ctx=rrlib.Context(kernel_family=2,
                                                            implementation_id=101))
        assert host(counts).tolist() == [r // 2, r // 2]


@pytest.mark.parametrize("experts", [1, 8, 33, 64, 256, 639, 640, 1024])
@pytest.mark.parametrize("dist", ["uniform", "zipf", "one"])
@pytest.mark.parametrize("routes", [1, 1000, 4099, 100_003, 1 << 18, 1 << 20])
def test_histogram_scan_fused_exact(rrlib, oracle, cuda, experts, dist, routes):
    from raggedroute_b200.workloads import route_ids
    ids_np = route_ids(routes, experts, dist, seed=routes + experts)
    counts_ref = oracle.histogram(ids_np, experts)
    offsets_ref = oracle.exclusive_scan(counts_ref)
    ids = dev(ids_np, cuda)
    counts = torch.full((experts,), 12345, dtype=torch.int32, device=cuda)
    offsets = torch.full((experts + 1,), -5, dtype=torch.int32, device=cuda)
    rrlib.histogram_exclusive_scan(ids, counts, offsets, routes, experts)
    assert np.array_equal(host(counts), counts_ref)
    assert np.array_equal(host(offsets), offsets_ref)
    # Standalone histogram + scan (with a non-16-byte-aligned id slice).
    counts2 = torch.full((experts,), 7, dtype=torch.int32, device=cuda)
    rrlib.histogram(ids, counts2, routes, experts)
    assert np.array_equal(host(counts2), counts_ref)
    if routes > 1:
        c3 = torch.empty(experts, dtype=torch.int32, device=cuda)
        rrlib.histogram(ids[1:], c3, routes - 1, experts)
        assert np.array_equal(host(c3), oracle.histogram(ids_np[1:], experts))
    off2 = torch.empty(experts + 1, dtype=torch.int32, device=cuda)
    rrlib.exclusive_scan(counts2, off2, experts)
    assert np.array_equal(host(off2), offsets_ref)


@pytest.mark.parametrize("experts,dist", [(256, "uniform"), (1, "one"), (1024, "zipf")])
def test_histogram_scan_many_cta_path(rrlib, oracle, cuda, experts, dist):
    """Above 256K routes the fused operator and the histogram merge CTAs
    through global atomics (below, through one thread-block cluster)."""
    from raggedroute_b200.workloads import route_ids
    routes = (1 << 20) + 4093
    ids_np = route_ids(routes, experts, dist, seed=experts + 77)
    counts_ref = oracle.histogram(ids_np, experts)
    ids = dev(ids_np, cuda)
    counts = torch.full((experts,), 3, dtype=torch.int32, device=cuda)
    offsets = torch.full((experts + 1,), 3, dtype=torch.int32, device=cuda)
    rrlib.histogram_exclusive_scan(ids, counts, offsets, routes, experts)
    assert np.array_equal(host(counts), counts_ref)
    assert np.array_equal(host(offsets), oracle.exclusive_scan(counts_ref))
    counts2 = torch.full((experts,), 3, dtype=torch.int32, device=cuda)
    rrlib.histogram(ids, counts2, routes, experts)
    assert np.array_equal(host(counts2), counts_ref)


def test_scan_in_place_alias(rrlib, oracle, cuda):
    # src/scan/cuda_naive/baseline.cu:20-22: counts and offsets may alias.
    counts_np = np.array([3, 0, 5, 1, 7], np.int32)
    buf = torch.zeros(6, dtype=torch.int32, device=cuda)
    buf[:5] = dev(counts_np, cuda)
    rrlib.exclusive_scan(buf[:5], buf, 5)
    assert host(buf).tolist() == oracle.exclusive_scan(counts_np).tolist()


def test_fused_scan_rejects_overlap(rrlib, cuda):
    buf = torch.zeros(16, dtype=torch.int32, device=cuda)
    with pytest.raises(rrlib.RaggedRouteError) as ei:
        rrlib.histogram_exclusive_scan(buf[:4], buf[2:6], buf[8:13], 4, 4)
    assert ei.value.code == rrlib.StatusCode.INVALID_ARGUMENT


# ---- token_permute ----------------------------------------------------------------

def _permute_case(rrlib, oracle, cuda, tokens, experts, top_k, hidden, dist="uniform",
                  misalign=False, seed=0):
    from raggedroute_b200.workloads import route_ids
    rng = np.random.default_rng(seed + tokens)
    x_np = rng.uniform(-1, 1, (tokens, hidden)).astype(np.float32)
    ids_np = route_ids(tokens * top_k, experts, dist, seed=seed + 1)
    offsets_np = oracle.exclusive_scan(oracle.histogram(ids_np, experts))
    xp_ref, pos_ref, sr_ref, cur_ref = oracle.stable_permute(x_np, ids_np, offsets_np, experts,
                                                             top_k)
    routes = tokens * top_k
    shift = 1 if misalign else 0
    xbuf = torch.empty(tokens * hidden + shift, dtype=torch.float32, device=cuda)
    xbuf[shift:] = dev(x_np.reshape(-1), cuda)
    x = xbuf[shift:]
    xpbuf = torch.full((routes * hidden + shift,), NAN, dtype=torch.float32, device=cuda)
    xp = xpbuf[shift:]
    pos = torch.full((routes,), -9, dtype=torch.int32, device=cuda)
    sr = torch.full((routes,), -9, dtype=torch.int32, device=cuda)
    ws_bytes = rrlib.token_permute_workspace_size(tokens, experts, top_k, hidden)
    ws = torch.full((max(ws_bytes, 4) // 4,), 99, dtype=torch.int32, device=cuda)
    rrlib.token_permute(x, dev(ids_np, cuda), dev(offsets_np, cuda), xp, pos, sr, tokens,
                        experts, top_k, hidden, ws)
    assert np.array_equal(host(pos), pos_ref)
    assert np.array_equal(host(sr), sr_ref)
    assert np.array_equal(host(ws)[:experts], cur_ref)
    got = host(xp).reshape(routes, hidden)
    assert np.array_equal(got.view(np.uint32), xp_ref.view(np.uint32))


def test_permute_kat(rrlib, oracle, cuda):
    # tests/operator_api_tests.cpp:734-804 with stale cursors {99,99}.
    x = dev(np.array([1, 2, 3, 4], np.float32), cuda)
    ids = dev(np.array([0, 1, 0, 1], np.int32), cuda)
    offsets = dev(np.array([0, 2, 4], np.int32), cuda)
    xp = torch.empty(8, device=cuda)
    pos = torch.empty(4, dtype=torch.int32, device=cuda)
    sr = torch.empty(4, dtype=torch.int32, device=cuda)
    assert rrlib.token_permute_workspace_size(2, 2, 2, 2) == 8
    for impl in range(0, 11):
        cursors = dev(np.array([99, 99], np.int32), cuda)
        ctx = rrlib.Context(kernel_family=2 if impl else 0, implementation_id=impl)
        rrlib.token_permute(x, ids, offsets, xp, pos, sr, 2, 2, 2, 2, cursors, ctx=ctx)
        assert host(cursors).tolist() == [2, 2]
        assert host(pos).tolist() == [0, 2, 1, 3]
        assert host(sr).tolist() == [0, 2, 1, 3]
        assert host(xp).tolist() == [1, 2, 3, 4, 1, 2, 3, 4]


def test_permute_workspace_contract(rrlib, cuda):
    # tests/operator_api_tests.cpp:303-315
    assert rrlib.token_permute_workspace_size(1, 2, 1, 0) == 8
    ids = torch.zeros(1, dtype=torch.int32, device=cuda)
    with pytest.raises(rrlib.RaggedRouteError) as ei:
        rrlib.token_permute(None, ids, ids, None, ids, None, 1, 2, 1, 0, None)
    assert ei.value.code == rrlib.StatusCode.INSUFFICIENT_WORKSPACE


@pytest.mark.parametrize("tokens,experts,top_k,hidden", [
    (1, 2, 1, 4), (5, 4, 2, 7), (128, 8, 2, 64), (129, 8, 2, 64), (1000, 64, 2, 128),
    (4096, 64, 2, 256), (3000, 256, 4, 33), (20000, 1024, 2, 16), (777, 3, 3, 1),
])
def test_permute_stable_exact(rrlib, oracle, cuda, tokens, experts, top_k, hidden):
    _permute_case(rrlib, oracle, cuda, tokens, experts, top_k, hidden)


@pytest.mark.parametrize("dist", ["zipf", "one"])
def test_permute_skewed(rrlib, oracle, cuda, dist):
    _permute_case(rrlib, oracle, cuda, 50_000, 64, 2, 32, dist=dist)


def test_permute_misaligned(rrlib, oracle, cuda):
    _permute_case(rrlib, oracle, cuda, 3000, 16, 2, 64, misalign=True)


def test_permute_c3_full_size_properties(rrlib, oracle, cuda):
    """C3 at full size: 1,048,576 routes, K=128, E=256 Zipf(1.5). route_pos is
    compared exactly with the vectorised oracle; rows through a checksum and a
    sampled exact check."""
    from raggedroute_b200.workloads import route_ids
    tokens, experts, hidden = 1 << 19, 256, 128
    ids_np = route_ids(2 * tokens, experts, "zipf", seed=2)
    offsets_np = oracle.exclusive_scan(oracle.histogram(ids_np, experts))
    pos_ref = oracle.stable_route_pos(ids_np, offsets_np, experts)
    x = torch.rand(tokens, hidden, device=cuda) * 2 - 1
    xp = torch.empty(2 * tokens, hidden, device=cuda)
    pos = torch.empty(2 * tokens, dtype=torch.int32, device=cuda)
    sr = torch.empty(2 * tokens, dtype=torch.int32, device=cuda)
    ws = torch.empty(rrlib.token_permute_workspace_size(tokens, experts, 2, hidden) // 4 + 1,
                     dtype=torch.int32, device=cuda)
    ids = dev(ids_np, cuda)
    rrlib.token_permute(x, ids, dev(offsets_np, cuda), xp, pos, sr, tokens, experts, 2, hidden, ws)
    assert np.array_equal(host(pos), pos_ref)
    assert np.array_equal(host(ws)[:experts], oracle.histogram(ids_np, experts))
    # Inverse map and row copies.
    sr_np = host(sr)
    assert np.array_equal(sr_np[pos_ref], np.arange(2 * tokens))
    src_tok = torch.as_tensor(sr_np // 2, device=cuda, dtype=torch.long)
    assert torch.equal(xp, x[src_tok])


def test_permute_low_level_launcher(rrlib, oracle, cuda):
    """ops::launch_token_permute_naive: cursors accumulate, stable order."""
    import ctypes
    lib = rrlib.lib()
    tokens, experts, top_k, hidden = 3000, 32, 2, 20
    rng = np.random.default_rng(5)
    ids_np = rng.integers(0, experts, tokens * top_k).astype(np.int32)
    offsets_np = oracle.exclusive_scan(oracle.histogram(ids_np, experts))
    x_np = rng.uniform(-1, 1, (tokens, hidden)).astype(np.float32)
    xp_ref, pos_ref, sr_ref, cur_ref = oracle.stable_permute(x_np, ids_np, offsets_np, experts,
                                                             top_k)
    x, ids, off = dev(x_np, cuda), dev(ids_np, cuda), dev(offsets_np, cuda)
    cursors = torch.zeros(experts, dtype=torch.int32, device=cuda)
    xp = torch.empty(tokens * top_k, hidden, device=cuda)
    pos = torch.empty(tokens * top_k, dtype=torch.int32, device=cuda)
    sr = torch.empty(tokens * top_k, dtype=torch.int32, device=cuda)
    rc = lib.rr_launch_token_permute_naive(x.data_ptr(), ids.data_ptr(), off.data_ptr(),
                                           cursors.data_ptr(), xp.data_ptr(), pos.data_ptr(),
                                           sr.data_ptr(), tokens, top_k, hidden,
                                           ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    assert np.array_equal(host(pos), pos_ref)
    assert np.array_equal(host(sr), sr_ref)
    assert np.array_equal(host(cursors), cur_ref)
    assert np.array_equal(host(xp), xp_ref)


# ---- unpermute --------------------------------------------------------------------

@pytest.mark.parametrize("tokens,top_k,output", [(1, 1, 1), (7, 2, 5), (4096, 2, 1024),
                                                 (100, 4, 128), (33, 8, 33), (50, 40, 12)])
def test_unpermute_parity(rrlib, oracle, cuda, tokens, top_k, output):
    rng = np.random.default_rng(tokens * 100 + output)
    routes = tokens * top_k
    yp = rng.uniform(-1, 1, (routes, output)).astype(np.float32)
    pos = rng.permutation(routes).astype(np.int32)
    rw = rng.uniform(0, 1, routes).astype(np.float32)
    y = torch.full((tokens, output), NAN, device=cuda)
    rrlib.unpermute(dev(yp, cuda), dev(pos, cuda), dev(rw, cuda), y, tokens, top_k, output)
    ref = oracle.unpermute_f64(yp, pos, rw, top_k)
    ok, err, rel = oracle.compare_floating(host(y), ref, 1e-6, 1e-5)
    assert ok, (err, rel)


# ---- GEMMs ------------------------------------------------------------------------

def _gemm_bound_ok(oracle, got, a, b, ref, k):
    bound = oracle.gemm_error_bound(a, b, k)
    err = np.abs(got.astype(np.float64) - ref)
    assert np.all(err <= bound), float((err - bound).max())
    assert oracle.normwise_rel_error(got, ref) <= 1e-5


def test_dense_kat(rrlib, cuda):
    a = dev(np.array([[1, 2], [3, 4]], np.float32), cuda)
    b = dev(np.array([[5, 6], [7, 8]], np.float32), cuda)
    c = torch.empty(2, 2, device=cuda)
    rrlib.dense_gemm(a, b, c, 2, 2, 2)
    assert host(c).reshape(-1).tolist() == [19.0, 22.0, 43.0, 50.0]


def test_dense_k0_writes_zeros(rrlib, cuda):
    c = torch.full((2, 2), 5.0, device=cuda)
    rrlib.dense_gemm(None, None, c, 2, 2, 0)
    assert host(c).reshape(-1).tolist() == [0.0] * 4


@pytest.mark.parametrize("m,n,k", [(1, 1, 1), (5, 3, 7), (512, 32, 256), (4096, 64, 256),
                                   (1000, 128, 4096), (333, 40, 100)])
def test_dense_parity(rrlib, oracle, cuda, m, n, k):
    rng = np.random.default_rng(m + n + k)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.normal(0, 1 / math.sqrt(k), (k, n)).astype(np.float32)
    c = torch.empty(m, n, device=cuda)
    rrlib.dense_gemm(dev(a, cuda), dev(b, cuda), c, m, n, k)
    _gemm_bound_ok(oracle, host(c), a, b, oracle.dense_gemm_f64(a, b), k)


def _grouped_case(rrlib, oracle, cuda, sizes, hidden, output, seed=0, check_rows=None):
    rng = np.random.default_rng(seed)
    sizes = np.asarray(sizes, np.int32)
    experts = sizes.size
    offsets = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int32)
    routes = int(offsets[-1])
    x = rng.uniform(-1, 1, (routes, hidden)).astype(np.float32)
    w = rng.normal(0, 1 / math.sqrt(max(hidden, 1)), (experts, hidden, output)).astype(np.float32)
    y = torch.full((routes, output), NAN, device=cuda)
    rrlib.grouped_gemm(dev(x, cuda), dev(w, cuda), dev(offsets, cuda), y, experts, hidden, output,
                       max(routes, 1))
    got = host(y)
    ref = oracle.grouped_gemm_f64(x, w, offsets)
    for e in range(experts):
        seg = slice(offsets[e], offsets[e + 1])
        if offsets[e + 1] > offsets[e]:
            _gemm_bound_ok(oracle, got[seg], x[seg], w[e], ref[seg], hidden)


@pytest.mark.parametrize("sizes,hidden,output", [
    ([3], 5, 7), ([0, 5, 0, 9], 7, 5), ([17, 1, 130, 0, 64], 64, 64),
    ([1000, 3, 0, 257], 256, 128), ([129] * 8, 128, 1408 // 8),
])
def test_grouped_parity(rrlib, oracle, cuda, sizes, hidden, output):
    _grouped_case(rrlib, oracle, cuda, sizes, hidden, output)


def test_grouped_c4_sizes(rrlib, oracle, cuda):
    """C4 group structure (Zipf 1.1, 6 forced-empty experts, no size a
    multiple of 16) at reduced K/N so the FP64 oracle stays fast."""
    from raggedroute_b200.workloads import c4_group_sizes
    sizes = c4_group_sizes(routes=4096)
    _grouped_case(rrlib, oracle, cuda, sizes, 256, 256, seed=3)


def test_grouped_k0_and_noop(rrlib, cuda):
    # tests/correctness_framework_tests.cpp:258-275
    offsets = dev(np.array([0, 2], np.int32), cuda)
    y = torch.full((2, 2), 3.0, device=cuda)
    rrlib.grouped_gemm(None, None, offsets, y, 1, 0, 2, 2)
    assert host(y).reshape(-1).tolist() == [0.0] * 4
    y.fill_(3.0)
    rrlib.grouped_gemm(None, None, offsets, y, 1, 0, 2, 0)  # max_expert_tokens = 0: no-op
    assert host(y).reshape(-1).tolist() == [3.0] * 4
