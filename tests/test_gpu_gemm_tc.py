"""tcgen05 GEMM engines (3xTF32 split; mixed TF32 + bfloat16 split of the
CTA-pair grouped GEMM from K = 128 up): accuracy against the FP64 oracle.

Tolerance: the reference's accumulation-aware FP32 bound
4*gamma_K*sum|a||b| + 1e-7 (src/correctness/reference_validation.cpp:70-115)
elementwise, AND a normwise relative error <= 1e-5.
Shapes cover ragged and empty groups, partial m/n/k tiles, groups shorter than
one tile at the start of the buffer, N > 256 and K up to 4096. Every case also
asserts that the engine selected was tcgen05 and that no bounded wait timed
out (device error word 0).
"""
from __future__ import annotations

import ctypes
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def dev(a, device):
    return torch.as_tensor(np.ascontiguousarray(a)).to(device)


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def device_error_word(rrlib) -> int:
    w = ctypes.c_uint32(0)
    st = rrlib.lib().rr_consume_device_error(
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), ctypes.byref(w))
    assert st.code == 0
    return int(w.value)


def check(oracle, got, a, b, ref, k):
    bound = oracle.gemm_error_bound(a, b, k)
    err = np.abs(got.astype(np.float64) - ref)
    assert np.all(err <= bound), float((err - bound).max())
    rel = oracle.normwise_rel_error(got, ref)
    assert rel <= 1e-5, rel
    return rel


@pytest.mark.parametrize("m,n,k", [(128, 256, 16), (1, 4, 4), (100, 36, 20), (300, 1408, 64),
                                   (4096, 128, 256), (512, 32, 256), (777, 260, 4096)])
def test_dense_tc(rrlib, oracle, cuda, m, n, k):
    rng = np.random.default_rng(m * 7 + n + k)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.normal(0, 1 / math.sqrt(k), (k, n)).astype(np.float32)
    da, db = dev(a, cuda), dev(b, cuda)
    c = torch.full((m, n), float("nan"), device=cuda)
    assert rrlib.grouped_gemm_engine(da, db, c, k, n) == \
        ("tcgen05_mixed" if k >= 128 else "tcgen05_3xtf32")
    rrlib.dense_gemm(da, db, c, m, n, k)
    check(oracle, host(c), a, b, oracle.dense_gemm_f64(a, b), k)
    assert device_error_word(rrlib) == 0


@pytest.mark.parametrize("sizes,k,n", [
    ([128], 16, 256),
    ([1, 0, 0, 5, 127, 129, 0, 300], 64, 96),
    ([0, 0, 17], 40, 1408),
    ([2000, 7, 0, 513], 512, 384),
    ([64] * 16, 4096, 128),
])
def test_grouped_tc(rrlib, oracle, cuda, sizes, k, n):
    rng = np.random.default_rng(len(sizes) * 31 + k + n)
    sizes = np.asarray(sizes, np.int32)
    e = sizes.size
    offsets = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int32)
    r = int(offsets[-1])
    x = rng.uniform(-1, 1, (r, k)).astype(np.float32)
    w = rng.normal(0, 1 / math.sqrt(k), (e, k, n)).astype(np.float32)
    dx, dw = dev(x, cuda), dev(w, cuda)
    y = torch.full((r, n), float("nan"), device=cuda)
    assert rrlib.grouped_gemm_engine(dx, dw, y, k, n) == \
        ("tcgen05_mixed" if k >= 128 else "tcgen05_3xtf32")
    rrlib.grouped_gemm(dx, dw, dev(offsets, cuda), y, e, k, n, r)
    got = host(y)
    ref = oracle.grouped_gemm_f64(x, w, offsets)
    for i in range(e):
        s = slice(offsets[i], offsets[i + 1])
        if offsets[i + 1] > offsets[i]:
            check(oracle, got[s], x[s], w[i], ref[s], k)
    assert not np.isnan(got).any()
    assert device_error_word(rrlib) == 0


@pytest.mark.parametrize("k", [124, 128, 132, 144, 1040])
def test_grouped_tc_split_boundary_and_worst_mantissas(rrlib, oracle, cuda, k):
    """K on both sides of the mixed split's threshold (124: 3xTF32; 128 and
    up: TF32 hi.hi plus bfloat16 corrections; 132 and 1040 end in a partial
    k-block; 1040 = two full 512-chunks plus one k-block), with operands whose
    split errors are largest: half the A values have all 13 low mantissa bits
    set (lo(A) just under one TF32 ulp of A, the largest truncation
    remainder), half the W values sit one bit off a TF32 rounding tie, so
    lo(W) is close to half an ulp and its bfloat16 rounding is exercised at
    every exponent. Elementwise within the accumulation-aware bound and 1e-5
    normwise against FP64."""
    rng = np.random.default_rng(k)
    sizes = np.asarray([300, 1, 0, 257], np.int32)
    e, n = sizes.size, 272
    offsets = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int32)
    r = int(offsets[-1])
    x = rng.uniform(-1, 1, (r, k)).astype(np.float32)
    xb = x.view(np.uint32)
    sel = rng.random((r, k)) < 0.5
    xb[sel] |= np.uint32(0x1FFF)
    w = (rng.normal(0, 1, (e, k, n)) * np.exp2(rng.integers(-20, 4, (e, k, n)))).astype(np.float32)
    wb = w.view(np.uint32)
    sel = rng.random((e, k, n)) < 0.5
    wb[sel] = (wb[sel] & np.uint32(0xFFFFE000)) | np.uint32(0x0FFF)   # just below a tie
    dx, dw = dev(x, cuda), dev(w, cuda)
    y = torch.full((r, n), float("nan"), device=cuda)
    rrlib.grouped_gemm(dx, dw, dev(offsets, cuda), y, e, k, n, r)
    got = host(y)
    ref = oracle.grouped_gemm_f64(x, w, offsets)
    for i in range(e):
        lo, hi = offsets[i], offsets[i + 1]
        if hi > lo:
            check(oracle, got[lo:hi], x[lo:hi], w[i], ref[lo:hi], k)
    assert device_error_word(rrlib) == 0


@pytest.mark.parametrize("k", [64, 256])
def test_grouped_tc_extreme_magnitudes(rrlib, oracle, cuda, k):
    """Operands across the FP32 range through both splits (K = 64: 3xTF32;
    K = 256: the mixed split with bfloat16 corrections): rows holding values
    up to 3.4e38 (beyond the largest finite bfloat16, 3.39e38) against
    weights that are exact in TF32 (their lo part is 0, so an unsaturated
    bfloat16 rounding of the large value would give inf * 0 = NaN in a
    correction product), rows of subnormals, of 1e-30 and of zeros, mixed
    with ordinary rows in the same tiles. Every output whose FP64 value is
    finite in FP32 must be finite and within the accumulation-aware bound."""
    rng = np.random.default_rng(k)
    sizes = np.asarray([150, 0, 90], np.int32)
    e, n = sizes.size, 40
    offsets = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int32)
    r = int(offsets[-1])
    x = rng.uniform(-1, 1, (r, k)).astype(np.float32)
    # Weights exact in TF32: multiples of 2^-8 in [-1, 1).
    w = (rng.integers(-256, 256, (e, k, n)) / 256.0).astype(np.float32)
    big = np.float32(3.4e38)
    x[3, :] = 0.0
    x[3, 5] = big                       # one huge term per output
    x[4, :] = 0.0
    x[4, 0], x[4, 1] = big, -big        # huge terms that cancel exactly... or not
    x[7, :] = rng.uniform(-1, 1, k).astype(np.float32) * np.float32(1e-40)  # subnormals
    x[8, :] = rng.uniform(-1, 1, k).astype(np.float32) * np.float32(1e-30)
    x[9, :] = 0.0
    x[160, :] = 0.0
    x[160, 7] = np.float32(-3.39e38)
    w[0, 5, :] = 0.25                   # finite products 8.5e37 for row 3
    dx, dw = dev(x, cuda), dev(w, cuda)
    y = torch.full((r, n), float("nan"), device=cuda)
    rrlib.grouped_gemm(dx, dw, dev(offsets, cuda), y, e, k, n, r)
    got = host(y)
    ref = oracle.grouped_gemm_f64(x, w, offsets)
    finite = np.abs(ref) < np.float64(np.finfo(np.float32).max)
    assert np.isfinite(got[finite]).all(), np.argwhere(~np.isfinite(got) & finite)[:8]
    for i in range(e):
        lo, hi = offsets[i], offsets[i + 1]
        if hi > lo:
            bound = oracle.gemm_error_bound(x[lo:hi], w[i], k)
            err = np.abs(got[lo:hi].astype(np.float64) - ref[lo:hi])
            ok = ~finite[lo:hi] | (err <= bound)
            assert ok.all(), np.argwhere(~ok)[:8]
    assert device_error_word(rrlib) == 0


@pytest.mark.parametrize("n", [8, 20, 40, 264, 1408])
def test_grouped_tc_half_tail_tiles(rrlib, oracle, cuda, n):
    """A last m-tile of an expert that stores at most 128 rows runs as an
    M = 128 pair MMA whose accumulator is folded across the TMEM lanes (64
    rows per CTA, columns [0, n/2) in lanes 0-63 and [n/2, n) in lanes
    64-127). Remainders 1, 64, 127, 128 of a 256-row tile take it, 129 and
    255 do not; every width, including half widths that are not a multiple
    of 16 (n = 40: 24 columns per half) and a 8-column last n-tile."""
    sizes = np.array([1, 64, 127, 128, 129, 255, 257, 384, 385, 612, 0, 3], np.int32)
    k = 64
    rng = np.random.default_rng(n)
    e = sizes.size
    offsets = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int32)
    r = int(offsets[-1])
    x = rng.uniform(-1, 1, (r, k)).astype(np.float32)
    w = rng.normal(0, 1 / math.sqrt(k), (e, k, n)).astype(np.float32)
    dx, dw = dev(x, cuda), dev(w, cuda)
    y = torch.full((r + 8, n), float("nan"), device=cuda)
    rrlib.grouped_gemm(dx, dw, dev(offsets, cuda), y, e, k, n, r)
    got = host(y)
    ref = oracle.grouped_gemm_f64(x, w, offsets)
    for i in range(e):
        s = slice(offsets[i], offsets[i + 1])
        if offsets[i + 1] > offsets[i]:
            check(oracle, got[s], x[s], w[i], ref[s], k)
    assert not np.isnan(got[:r]).any()
    assert np.isnan(got[r:]).all()
    assert device_error_word(rrlib) == 0


def test_grouped_tc_rows_outside_segments_untouched(rrlib, cuda):
    """Rows past offsets[E] keep their previous contents."""
    k, n = 32, 64
    offsets = np.array([0, 50, 50, 90], np.int32)
    x = torch.rand(128, k, device=cuda)
    w = torch.rand(3, k, n, device=cuda)
    y = torch.full((128, n), 7.0, device=cuda)
    rrlib.grouped_gemm(x, w, dev(offsets, cuda), y, 3, k, n, 90)
    torch.cuda.synchronize()
    assert torch.all(y[90:] == 7.0)
    assert device_error_word(rrlib) == 0


def test_grouped_tc_c4_full_size_sampled(rrlib, oracle, cuda):
    """C4 at full size (R=32768, E=64, K=N=1024, Zipf 1.1 groups with 6
    empty experts, no size a multiple of 16): every expert's first, last and
    a seeded sample of rows checked against the FP64 oracle."""
    from raggedroute_b200.workloads import c4_group_sizes, offsets_from_sizes
    sizes = c4_group_sizes()
    offsets = offsets_from_sizes(sizes)
    r, e, k, n = 32768, 64, 1024, 1024
    g = torch.Generator(device=cuda)
    g.manual_seed(3)
    x = torch.rand(r, k, generator=g, device=cuda) * 2 - 1
    w = torch.randn(e, k, n, generator=g, device=cuda) / math.sqrt(32.0 * 32.0)
    y = torch.full((r, n), float("nan"), device=cuda)
    rrlib.grouped_gemm(x, w, dev(offsets, cuda), y, e, k, n, r)
    rng = np.random.default_rng(3)
    rows = set()
    for i in range(e):
        if sizes[i] > 0:
            rows.update({int(offsets[i]), int(offsets[i + 1] - 1)})
    rows.update(rng.integers(0, r, 200).tolist())
    rows = np.array(sorted(rows))
    xs = host(x)[rows]
    ws = host(w)
    ys = host(y)[rows]
    expert_of = np.searchsorted(offsets, rows, side="right") - 1
    for j, row in enumerate(rows):
        ei = expert_of[j]
        ref = xs[j].astype(np.float64) @ ws[ei].astype(np.float64)
        bound = oracle.gemm_error_bound(xs[j][None, :], ws[ei], k)[0]
        assert np.all(np.abs(ys[j] - ref) <= bound)
    assert oracle.normwise_rel_error(ys, np.stack([xs[j].astype(np.float64) @ ws[expert_of[j]]
                                                   for j in range(len(rows))])) <= 1e-5
    assert not torch.isnan(y).any()
    assert device_error_word(rrlib) == 0


def test_grouped_tc_c5_shape_sampled(rrlib, oracle, cuda):
    """The C5 grouped GEMM at its full shape (R=131072 rows, E=128, K=4096,
    N=1408) with ragged C5-like groups (Zipf 1.0, 4 forced-empty experts, no
    size a multiple of 16): every expert's first and last row and 300 seeded
    rows against the FP64 oracle, elementwise within the accumulation-aware
    bound and normwise within 1e-5."""
    from raggedroute_b200.workloads import c4_group_sizes, offsets_from_sizes
    r, e, k, n = 131072, 128, 4096, 1408
    sizes = c4_group_sizes(routes=r, experts=e, empty=4, s=1.0, seed=4)
    offsets = offsets_from_sizes(sizes)
    g = torch.Generator(device=cuda)
    g.manual_seed(4)
    x = torch.randn(r, k, generator=g, device=cuda)
    w = torch.randn(e, k, n, generator=g, device=cuda) / 64.0
    y = torch.full((r, n), float("nan"), device=cuda)
    rrlib.grouped_gemm(x, w, dev(offsets, cuda), y, e, k, n, r)
    rng = np.random.default_rng(4)
    rows = set(rng.integers(0, r, 300).tolist())
    for i in range(e):
        if sizes[i] > 0:
            rows.update({int(offsets[i]), int(offsets[i + 1] - 1)})
    rows = np.array(sorted(rows))
    expert_of = np.searchsorted(offsets, rows, side="right") - 1
    xs = host(x[torch.from_numpy(rows).to(cuda)])
    ys = host(y[torch.from_numpy(rows).to(cuda)])
    ref = np.empty((rows.size, n), np.float64)
    for ei in np.unique(expert_of):
        sel = np.nonzero(expert_of == ei)[0]
        wi = host(w[int(ei)])
        ref[sel] = xs[sel].astype(np.float64) @ wi.astype(np.float64)
        bound = oracle.gemm_error_bound(xs[sel], wi, k)
        assert np.all(np.abs(ys[sel] - ref[sel]) <= bound), int(ei)
    rel = oracle.normwise_rel_error(ys, ref)
    assert rel <= 1e-5, rel
    assert not torch.isnan(y).any()
    assert device_error_word(rrlib) == 0


@pytest.mark.parametrize("m,n,k", [(40000, 128, 256), (37999, 100, 64), (65536, 128, 128)])
def test_dense_tc_two_tiles_per_cta(rrlib, oracle, cuda, m, n, k):
    """Router-shaped GEMMs (N <= 128, at least one wave of 256-row tiles);
    ragged row counts leave a shifted last tile. By default they run the
    narrow kernel; the engine's two 128-row m-tiles per CTA (sharing each B
    tile) run under RAGGEDROUTE_B200_NARROW_DENSE=0 (test_gpu_engines)."""
    rng = np.random.default_rng(m + n)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.normal(0, 1 / math.sqrt(k), (k, n)).astype(np.float32)
    da, db = dev(a, cuda), dev(b, cuda)
    c = torch.full((m, n), float("nan"), device=cuda)
    rrlib.dense_gemm(da, db, c, m, n, k)
    got = host(c)
    ref = oracle.dense_gemm_f64(a, b)
    rows = rng.choice(m, 2048, replace=False)
    rows[:2] = [0, m - 1]
    check(oracle, got[rows], a[rows], b, ref[rows], k)
    assert oracle.normwise_rel_error(got, ref) <= 1e-5
    assert device_error_word(rrlib) == 0


@pytest.mark.parametrize("m,n,k", [(65536, 128, 4096), (50003, 60, 512)])
def test_dense_narrow_router_shapes(rrlib, oracle, cuda, m, n, k):
    """Dense GEMMs with N <= 128 take the transposed narrow kernel (token tiles of 224 at C5's router shape,
    65536 x 4096 x 128; a ragged row count and N = 60 with a shifted last
    tile): 2048 sampled rows plus the first and last against the FP64
    oracle, elementwise within the accumulation-aware bound and normwise
    within 1e-5."""
    g = torch.Generator(device=cuda)
    g.manual_seed(m + n)
    a = torch.randn(m, k, generator=g, device=cuda)
    b = torch.randn(k, n, generator=g, device=cuda) / math.sqrt(k)
    c = torch.full((m, n), float("nan"), device=cuda)
    rrlib.dense_gemm(a, b, c, m, n, k)
    torch.cuda.synchronize()
    assert not torch.isnan(c).any()
    rng = np.random.default_rng(m)
    rows = np.unique(np.concatenate([[0, m - 1], rng.choice(m, 2048, replace=False)]))
    sel = torch.from_numpy(rows).to(cuda)
    a_s, c_s, b_h = host(a[sel]), host(c[sel]), host(b)
    check(oracle, c_s, a_s, b_h, oracle.dense_gemm_f64(a_s, b_h), k)
    assert device_error_word(rrlib) == 0


@pytest.mark.parametrize("m,n,k", [(65536, 128, 4096), (40000, 60, 512)])
def test_dense_narrow_batch_independent(rrlib, cuda, m, n, k):
    """The router GEMM's result for a row does not depend on the batch the
    row arrives in: rows computed inside the whole batch (token tiles of 224
    or 144 rows) and inside slices of 8192, 300, 37 and 1 rows (tiles of 32)
    are the same bits. The chunked host-memory chain relies on this."""
    g = torch.Generator(device=cuda)
    g.manual_seed(m + 7 * n)
    a = torch.randn(m, k, generator=g, device=cuda)
    b = torch.randn(k, n, generator=g, device=cuda) / math.sqrt(k)
    c = torch.full((m, n), float("nan"), device=cuda)
    rrlib.dense_gemm(a, b, c, m, n, k)
    for start, rows in [(1000, 8192), (m - 300, 300), (5, 37), (m - 1, 1), (0, 1)]:
        a_s = a[start:start + rows].contiguous()
        c_s = torch.full((rows, n), float("nan"), device=cuda)
        rrlib.dense_gemm(a_s, b, c_s, rows, n, k)
        torch.cuda.synchronize()
        assert torch.equal(c_s.view(torch.int32), c[start:start + rows].view(torch.int32)), \
            (start, rows)
    assert device_error_word(rrlib) == 0


def test_integer_tf32_rounding_matches_cvt(rrlib, cuda):
    """The split rounds to TF32 with integer adds on the bit pattern; it must
    equal cvt.rna.tf32.f32 for every non-NaN input: random bit patterns over
    the whole range plus the edge values (zeros, denormals, ties, the
    largest finite values, infinities)."""
    rng = np.random.default_rng(5)
    rnd = rng.integers(0, 2**32, 1 << 22, dtype=np.uint64)
    edges = []
    for m in (0, 1, 0xFFF, 0x1000, 0x1001, 0x1FFF, 0x2000, 0x3000, 0x7FF000, 0x7FFFFF):
        for e in (0, 1, 0x7E, 0x7F, 0x80, 0xFE):
            for sgn in (0, 1):
                edges.append((sgn << 31) | (e << 23) | m)
    edges += [0x7F800000, 0xFF800000, 0x7F7FFFFF, 0xFF7FFFFF, 0x7F7FF000, 0x7F7FEFFF]
    bits = np.concatenate([rnd, np.array(edges, dtype=np.uint64)]).astype(np.uint32)
    dbits = torch.from_numpy(bits.view(np.int32)).to(cuda)
    count = torch.zeros(1, dtype=torch.int64, device=cuda)
    st = rrlib.lib().rr_tf32_rounding_selfcheck(
        ctypes.c_void_p(dbits.data_ptr()), dbits.numel(), ctypes.c_void_p(count.data_ptr()),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st.code == 0
    torch.cuda.synchronize()
    assert int(count.item()) == 0
