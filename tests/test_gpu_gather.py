"""Row-gathering grouped GEMM (the reference's
launch_grouped_gemm_sm86_fp32_gather_v1 contract) and the gather option of
the chains. The gather GEMM runs the one-CTA tcgen05 engine with the 3xTF32
split (or the FP32 SIMT engine for shapes TMA cannot take); the default
grouped GEMM runs the CTA-pair engine, with the mixed split from K = 128 up.
So the GEMM that reads row r from x[sorted_route[r] / top_k] must equal the
GEMM over the materialised x_permuted bit for bit below K = 128, and hold
the FP32 contract against FP64 (accumulation-aware bound, 1e-5 normwise)
everywhere (shifted first tiles, empty experts); its bit-identity with the
3xTF32 pair engine at any K is checked in tests/test_gpu_engines.py. Every
chain run with gather_rows must give the same ids, positions and
permutation, an output within the FP32 contract, and leave x_permuted
untouched."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from route_ids import make_route_ids, make_route_weights

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("t,k,e,n,top_k", [(500, 256, 16, 192, 2), (1200, 128, 32, 1408, 4),
                                           (37, 20, 8, 36, 2), (300, 30, 8, 10, 2)])
def test_gather_gemm_equals_materialised(rrlib, oracle, cuda, t, k, e, n, top_k):
    rng = np.random.default_rng(t + k)
    x = torch.from_numpy(rng.uniform(-1, 1, (t, k)).astype(np.float32)).to(cuda)
    w = torch.from_numpy(rng.normal(0, 0.1, (e, k, n)).astype(np.float32)).to(cuda)
    ids = torch.from_numpy(make_route_ids(t, top_k, e, "zipf", 1.3, t)).to(cuda)
    rw = torch.from_numpy(make_route_weights(t, top_k, t)).to(cuda)
    buf = rrlib.RouteChainBuffers.allocate(t, top_k, k, e, n, cuda)
    rrlib.chain_from_route_ids(x, ids, rw, w, buf)  # materialised x_permuted + sorted_route
    torch.cuda.synchronize()
    r = t * top_k
    y_gather = torch.full((r, n), float("nan"), device=cuda)
    rrlib.grouped_gemm_gather(x, buf.sorted_route, top_k, w, buf.offsets, y_gather, r)
    torch.cuda.synchronize()
    if k < 128:
        assert torch.equal(y_gather.view(torch.int32), buf.y_permuted.view(torch.int32))
    xp = x.cpu().numpy()[buf.sorted_route.cpu().numpy() // top_k]
    offsets = buf.offsets.cpu().numpy()
    ref = oracle.grouped_gemm_f64(xp, w.cpu().numpy(), offsets)
    wn = w.cpu().numpy()
    for got in (y_gather, buf.y_permuted):
        g = got.cpu().numpy()
        for ex in range(e):
            lo, hi = offsets[ex], offsets[ex + 1]
            if hi > lo:
                bound = oracle.gemm_error_bound(xp[lo:hi], wn[ex], k)
                assert np.all(np.abs(g[lo:hi].astype(np.float64) - ref[lo:hi]) <= bound), ex
        assert oracle.normwise_rel_error(g, ref) <= 1e-5


def test_chains_with_gather_rows(rrlib, oracle, cuda):
    from raggedroute_b200.workloads import normal, zipf_log_bias
    t, k, e, n = 3000, 256, 64, 192
    x = normal((t, k), 1.0, 21, cuda)
    wr = normal((k, e), 1 / 16, 22, cuda)
    we = normal((e, k, n), 1 / 16, 23, cuda)
    bias = torch.from_numpy(zipf_log_bias(e, 1.0)).to(cuda)
    a = rrlib.ChainBuffers.allocate(t, k, e, n, cuda)
    b = rrlib.ChainBuffers.allocate(t, k, e, n, cuda)
    b.x_permuted.fill_(float("nan"))
    rrlib.chain_from_tokens(x, wr, we, a, logit_bias=bias)
    rrlib.chain_from_tokens(x, wr, we, b, logit_bias=bias, gather_rows=True)
    torch.cuda.synchronize()
    for name in ("expert_ids", "counts", "offsets", "route_pos"):
        assert torch.equal(getattr(a, name), getattr(b, name)), name
    y64 = oracle.chain_output_f64(x.cpu().numpy(), we.cpu().numpy(),
                                  a.expert_ids.cpu().numpy(), a.route_weights.cpu().numpy())
    for buf in (a, b):
        assert oracle.normwise_rel_error(buf.y.cpu().numpy(), y64) <= 1e-5
    assert torch.isnan(b.x_permuted).all()
    # chain_from_logits on the same logits: the same gather GEMM, same bits
    c = rrlib.ChainBuffers.allocate(t, k, e, n, cuda)
    rrlib.chain_from_logits(a.logits + bias, x, we, c, gather_rows=True)
    torch.cuda.synchronize()
    assert torch.equal(c.y.view(torch.int32), b.y.view(torch.int32))
    # post-route chain, top_k 4
    ids = torch.from_numpy(make_route_ids(t, 4, e, "zipf", 1.2, 5)).to(cuda)
    rw = torch.from_numpy(make_route_weights(t, 4, 5)).to(cuda)
    ra = rrlib.RouteChainBuffers.allocate(t, 4, k, e, n, cuda)
    rb = rrlib.RouteChainBuffers.allocate(t, 4, k, e, n, cuda)
    rrlib.chain_from_route_ids(x, ids, rw, we, ra)
    rrlib.chain_from_route_ids(x, ids, rw, we, rb, gather_rows=True)
    torch.cuda.synchronize()
    assert torch.equal(ra.sorted_route, rb.sorted_route)
    y64 = oracle.chain_output_f64(x.cpu().numpy(), we.cpu().numpy(), ids.cpu().numpy(),
                                  rw.cpu().numpy())
    for buf in (ra, rb):
        assert oracle.normwise_rel_error(buf.y.cpu().numpy(), y64) <= 1e-5


def test_unknown_chain_implementation_is_rejected(rrlib, cuda):
    from raggedroute_b200._lib import RaggedRouteError
    t, k, e, n = 16, 8, 4, 8
    buf = rrlib.ChainBuffers.allocate(t, k, e, n, cuda)
    x = torch.zeros(t, k, device=cuda)
    with pytest.raises(RaggedRouteError):
        rrlib.chain_from_tokens(x, torch.zeros(k, e, device=cuda), torch.zeros(e, k, n, device=cuda),
                                buf, ctx=rrlib.Context(implementation_id=7))
