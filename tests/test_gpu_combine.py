"""The unpermute fused into the grouped GEMM's epilogue, and the row-address
(scatter) epilogue, on one GPU.

* launch_unpermute equals the float32 oracle of its arithmetic bit for bit
  (rounded product, then round-to-nearest add with subnormal operands and
  results flushed to zero, rank order from 0.0f), subnormal-laden inputs
  included; and the FP64 reference value within the reference's tolerance.
* rr_grouped_gemm_combine equals rr_grouped_gemm followed by rr_unpermute bit
  for bit for top_k 1 and 2 (tcgen05 CTA-pair engine, and the FP32 SIMT
  engine for shapes TMA cannot take), with ragged and empty groups; top_k 4
  is refused.
* Every chain with fused_combine (alone, with gather_rows, with prepared
  weights) gives the same ids and positions as the unfused chain and leaves
  y_permuted untouched; y equals the unfused chain's bit for bit on the same
  GEMM engine (the gather and prepared options run the one-CTA 3xTF32
  engine, the default the CTA-pair engine with the mixed split from K = 128
  up, so across engines y is held to 1e-5 normwise against FP64); the post-route chain likewise for top_k 1
  and 2 and refuses top_k 4; also at the full C5 shape.
* rr_grouped_gemm_scatter stores each row at its packed address in one of
  several buffers (one of them not 16-byte aligned), bit-equal to the plain
  GEMM's row, and skips negative, out-of-range-buffer and out-of-range-row
  addresses.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from route_ids import make_route_ids, make_route_weights

pytestmark = pytest.mark.gpu


def bits(t: torch.Tensor) -> torch.Tensor:
    return t.contiguous().view(torch.int32)


def _routes(rrlib, cuda, t, k, e, n, top_k, seed, dist="zipf"):
    """Inputs of a grouped GEMM in permuted order: x_permuted, offsets and
    sorted_route from the library's own stable permute (through the
    post-route chain, whose y is the separate-unpermute result)."""
    rng = np.random.default_rng(seed)
    x = torch.from_numpy(rng.uniform(-1, 1, (t, k)).astype(np.float32)).to(cuda)
    w = torch.from_numpy(rng.normal(0, 0.1, (e, k, n)).astype(np.float32)).to(cuda)
    ids = torch.from_numpy(make_route_ids(t, top_k, e, dist, 1.3, seed)).to(cuda)
    rw = torch.from_numpy(make_route_weights(t, top_k, seed)).to(cuda)
    buf = rrlib.RouteChainBuffers.allocate(t, top_k, k, e, n, cuda)
    rrlib.chain_from_route_ids(x, ids, rw, w, buf)
    torch.cuda.synchronize()
    return x, w, ids, rw, buf


@pytest.mark.parametrize("tokens,top_k,output", [(1, 1, 4), (777, 2, 1408), (300, 2, 37),
                                                 (129, 4, 64), (50, 8, 12)])
def test_unpermute_bit_exact_against_ftz_oracle(rrlib, oracle, cuda, tokens, top_k, output):
    rng = np.random.default_rng(tokens * 13 + output)
    routes = tokens * top_k
    yp = rng.normal(0, 1, (routes, output)).astype(np.float32)
    # Plant subnormal values and products, and signed zeros, where the flush
    # decides the result.
    flat = yp.reshape(-1)
    pick = rng.choice(flat.size, max(1, flat.size // 7), replace=False)
    flat[pick[0::4]] = rng.uniform(-1, 1, pick[0::4].size).astype(np.float32) * np.float32(1e-38)
    flat[pick[1::4]] = -0.0
    flat[pick[2::4]] = np.float32(3e-39)
    pos = rng.permutation(routes).astype(np.int32)
    w = rng.uniform(0, 1, routes).astype(np.float32)
    w[rng.choice(routes, max(1, routes // 5), replace=False)] = np.float32(1e-30)
    y = torch.full((tokens, output), float("nan"), device=cuda)
    rrlib.unpermute(torch.from_numpy(yp).to(cuda), torch.from_numpy(pos).to(cuda),
                    torch.from_numpy(w).to(cuda), y, tokens, top_k, output)
    torch.cuda.synchronize()
    got = y.cpu().numpy()
    ref = oracle.unpermute_f32_ftz(yp, pos, w, top_k)
    assert np.array_equal(got.view(np.int32), ref.view(np.int32))
    # The reference's tolerance against the exact value
    # (benchmarks/adapters/unpermute_adapter.cpp:134).
    assert oracle.compare_floating(got, oracle.unpermute_f64(yp, pos, w, top_k), 1e-6, 1e-5)[0]


@pytest.mark.parametrize("t,k,e,n,top_k", [
    (2000, 256, 16, 192, 2),    # CTA-pair engine, ragged groups
    (1500, 128, 64, 1408, 2),   # N > 256: several column tiles, some experts empty
    (900, 64, 8, 256, 1),       # top_k 1
    (300, 30, 8, 10, 2),        # K, N not multiples of 4: FP32 SIMT engine
    (37, 20, 8, 36, 2),         # tiny, K not a multiple of 4
])
def test_grouped_gemm_combine_equals_gemm_then_unpermute(rrlib, cuda, t, k, e, n, top_k):
    x, w, ids, rw, buf = _routes(rrlib, cuda, t, k, e, n, top_k, t + n)
    r = t * top_k
    yp = torch.full((r, n), float("nan"), device=cuda)
    rrlib.grouped_gemm(buf.x_permuted, w, buf.offsets, yp, e, k, n, r)
    y_ref = torch.full((t, n), float("nan"), device=cuda)
    rrlib.unpermute(yp, buf.route_pos, rw, y_ref, t, top_k, n)
    y = torch.full((t, n), float("nan"), device=cuda)
    rrlib.grouped_gemm_combine(buf.x_permuted, w, buf.offsets, buf.sorted_route, rw, y, r, top_k)
    torch.cuda.synchronize()
    assert torch.equal(bits(y), bits(y_ref))
    assert torch.equal(bits(y), bits(buf.y))  # the route chain's own output


def test_grouped_gemm_combine_refuses_top_k_above_2(rrlib, cuda):
    from raggedroute_b200._lib import RaggedRouteError, StatusCode
    t, k, e, n = 64, 16, 4, 8
    x, w, ids, rw, buf = _routes(rrlib, cuda, t, k, e, n, 4, 3)
    y = torch.empty(t, n, device=cuda)
    with pytest.raises(RaggedRouteError) as info:
        rrlib.grouped_gemm_combine(buf.x_permuted, w, buf.offsets, buf.sorted_route, rw, y,
                                   t * 4, 4)
    assert info.value.code == StatusCode.UNSUPPORTED_KERNEL_VARIANT


def test_chains_with_fused_combine_are_bit_identical(rrlib, oracle, cuda):
    from raggedroute_b200.workloads import normal, zipf_log_bias
    t, k, e, n = 3000, 256, 64, 192
    x = normal((t, k), 1.0, 31, cuda)
    wr = normal((k, e), 1 / 16, 32, cuda)
    we = normal((e, k, n), 1 / 16, 33, cuda)
    bias = torch.from_numpy(zipf_log_bias(e, 1.0)).to(cuda)
    ref = rrlib.ChainBuffers.allocate(t, k, e, n, cuda)
    rrlib.chain_from_tokens(x, wr, we, ref, logit_bias=bias)
    for opts in (dict(fused_combine=True), dict(fused_combine=True, gather_rows=True)):
        b = rrlib.ChainBuffers.allocate(t, k, e, n, cuda)
        b.y_permuted.fill_(float("nan"))
        b.y.fill_(float("nan"))
        rrlib.chain_from_tokens(x, wr, we, b, logit_bias=bias, **opts)
        torch.cuda.synchronize()
        for name in ("expert_ids", "counts", "offsets", "route_pos"):
            assert torch.equal(getattr(ref, name), getattr(b, name)), (opts, name)
        if opts.get("gather_rows"):
            # Fused against unfused on the gather engine: same bits.
            u = rrlib.ChainBuffers.allocate(t, k, e, n, cuda)
            rrlib.chain_from_tokens(x, wr, we, u, logit_bias=bias, gather_rows=True)
            torch.cuda.synchronize()
            assert torch.equal(bits(u.y), bits(b.y)), opts
            y64 = oracle.chain_output_f64(x.cpu().numpy(), we.cpu().numpy(),
                                          ref.expert_ids.cpu().numpy(),
                                          ref.route_weights.cpu().numpy())
            assert oracle.normwise_rel_error(b.y.cpu().numpy(), y64) <= 1e-5, opts
        else:
            assert torch.equal(bits(ref.y), bits(b.y)), opts
        assert torch.isnan(b.y_permuted).all(), opts
    # chain_from_logits on the same logits
    c = rrlib.ChainBuffers.allocate(t, k, e, n, cuda)
    rrlib.chain_from_logits(ref.logits + bias, x, we, c, fused_combine=True)
    torch.cuda.synchronize()
    assert torch.equal(bits(c.y), bits(ref.y))
    # prepared expert weights: fused against the same chain unfused
    prep = rrlib.PreparedExpertWeights(we)
    p0 = rrlib.ChainBuffers.allocate(t, k, e, n, cuda)
    p1 = rrlib.ChainBuffers.allocate(t, k, e, n, cuda)
    rrlib.chain_from_tokens(x, wr, prep, p0, logit_bias=bias)
    rrlib.chain_from_tokens(x, wr, prep, p1, logit_bias=bias, fused_combine=True)
    torch.cuda.synchronize()
    assert torch.equal(bits(p0.y), bits(p1.y))


@pytest.mark.parametrize("top_k", [1, 2])
def test_route_chain_fused_combine(rrlib, cuda, top_k):
    t, k, e, n = 2500, 128, 32, 256
    x, w, ids, rw, a = _routes(rrlib, cuda, t, k, e, n, top_k, 40 + top_k)
    b = rrlib.RouteChainBuffers.allocate(t, top_k, k, e, n, cuda)
    b.y_permuted.fill_(float("nan"))
    rrlib.chain_from_route_ids(x, ids, rw, w, b, fused_combine=True)
    torch.cuda.synchronize()
    assert torch.equal(a.sorted_route, b.sorted_route)
    assert torch.equal(bits(a.y), bits(b.y))
    assert torch.isnan(b.y_permuted).all()


def test_route_chain_fused_combine_refuses_top_k_4(rrlib, cuda):
    from raggedroute_b200._lib import RaggedRouteError, StatusCode
    t, k, e, n = 64, 16, 8, 8
    x, w, ids, rw, a = _routes(rrlib, cuda, t, k, e, n, 4, 5)
    with pytest.raises(RaggedRouteError) as info:
        rrlib.chain_from_route_ids(x, ids, rw, w, a, fused_combine=True)
    assert info.value.code == StatusCode.UNSUPPORTED_KERNEL_VARIANT
    with pytest.raises(RaggedRouteError) as info:
        rrlib.chain_from_route_ids(x, ids, rw, w, a, ctx=rrlib.Context(implementation_id=8))
    assert info.value.code == StatusCode.UNSUPPORTED_KERNEL_VARIANT


def test_c5_chain_fused_combine_bit_identical(rrlib, cuda):
    """The full C5 shape (T=65536, K=4096, E=128, N=1408, log-Zipf router
    bias): fused and separate unpermute give the same y bit for bit."""
    from raggedroute_b200.workloads import C5, c5_inputs
    inp = c5_inputs(cuda)
    t, k, e, n = C5["tokens"], C5["hidden"], C5["experts"], C5["output"]
    a = rrlib.ChainBuffers.allocate(t, k, e, n, cuda)
    rrlib.chain_from_tokens(inp.x, inp.router_w, inp.expert_w, a, logit_bias=inp.logit_bias)
    torch.cuda.synchronize()
    y_ref = a.y.clone()
    a.y.fill_(float("nan"))
    rrlib.chain_from_tokens(inp.x, inp.router_w, inp.expert_w, a, logit_bias=inp.logit_bias,
                            fused_combine=True)
    torch.cuda.synchronize()
    assert torch.equal(bits(a.y), bits(y_ref))


def test_grouped_gemm_scatter(rrlib, cuda):
    t, k, e, n, top_k = 1000, 128, 16, 264, 2
    x, w, ids, rw, buf = _routes(rrlib, cuda, t, k, e, n, top_k, 77)
    r = t * top_k
    yp = torch.empty(r, n, device=cuda)
    rrlib.grouped_gemm(buf.x_permuted, w, buf.offsets, yp, e, k, n, r)
    # Three destination buffers; the third starts 4 bytes into its
    # allocation, so its rows are not 16-byte aligned.
    rows_per = r // 2 + 8
    dst = [torch.full((rows_per, n), float("nan"), device=cuda) for _ in range(2)]
    raw = torch.full((rows_per * n + 1,), float("nan"), device=cuda)
    dst.append(raw[1:].view(rows_per, n))
    bases = torch.tensor([d.data_ptr() for d in dst], dtype=torch.int64, device=cuda)
    rng = np.random.default_rng(9)
    # Distinct (buffer, row) pairs, so every stored row can be checked.
    pairs = rng.permutation(3 * rows_per)[:r]
    which, row = pairs // rows_per, pairs % rows_per
    addr = (which.astype(np.int64) << 40) | row.astype(np.int64)
    skip = rng.choice(r, 60, replace=False)
    addr[skip[:20]] = -1                                  # negative
    addr[skip[20:40]] = (np.int64(3) << 40) | 5           # buffer index out of range
    addr[skip[40:]] = (np.int64(1) << 40) | rows_per      # row at the limit
    rrlib.grouped_gemm_scatter(buf.x_permuted, w, buf.offsets,
                               torch.from_numpy(addr).to(cuda), bases, rows_per, r)
    torch.cuda.synchronize()
    got = [d.cpu().numpy() for d in dst]
    ypn = yp.cpu().numpy()
    written = [np.zeros(rows_per, bool) for _ in range(3)]
    keep = np.ones(r, bool)
    keep[skip] = False
    for i in np.nonzero(keep)[0]:
        b, q = int(which[i]), int(row[i])
        assert np.array_equal(got[b][q].view(np.int32), ypn[i].view(np.int32)), (i, b, q)
        written[b][q] = True
    for b in range(3):
        assert np.isnan(got[b][~written[b]]).all()
