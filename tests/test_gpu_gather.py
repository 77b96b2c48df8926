"""Row-gathering grouped GEMM (the reference's
launch_grouped_gemm_sm86_fp32_gather_v1 contract) and the gather option of
the chains: the GEMM that reads row r from x[sorted_route[r] / top_k] must
equal the GEMM over the materialised x_permuted bit for bit (tcgen05 and
FP32 SIMT engines, shifted first tiles, empty experts), and every chain run
with gather_rows must give the same ids, positions and output bit for bit
while leaving x_permuted untouched."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from route_ids import make_route_ids, make_route_weights

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("t,k,e,n,top_k", [(500, 256, 16, 192, 2), (1200, 128, 32, 1408, 4),
                                           (37, 20, 8, 36, 2), (300, 30, 8, 10, 2)])
def test_gather_gemm_equals_materialised(rrlib, cuda, t, k, e, n, top_k):
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
    assert torch.equal(y_gather.view(torch.int32), buf.y_permuted.view(torch.int32))


def test_chains_with_gather_rows_are_bit_identical(rrlib, cuda):
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
    assert torch.equal(a.y.view(torch.int32), b.y.view(torch.int32))
    assert torch.isnan(b.x_permuted).all()
    # chain_from_logits on the same logits
    c = rrlib.ChainBuffers.allocate(t, k, e, n, cuda)
    rrlib.chain_from_logits(a.logits + bias, x, we, c, gather_rows=True)
    torch.cuda.synchronize()
    assert torch.equal(c.y.view(torch.int32), a.y.view(torch.int32))
    # post-route chain, top_k 4
    ids = torch.from_numpy(make_route_ids(t, 4, e, "zipf", 1.2, 5)).to(cuda)
    rw = torch.from_numpy(make_route_weights(t, 4, 5)).to(cuda)
    ra = rrlib.RouteChainBuffers.allocate(t, 4, k, e, n, cuda)
    rb = rrlib.RouteChainBuffers.allocate(t, 4, k, e, n, cuda)
    rrlib.chain_from_route_ids(x, ids, rw, we, ra)
    rrlib.chain_from_route_ids(x, ids, rw, we, rb, gather_rows=True)
    torch.cuda.synchronize()
    assert torch.equal(ra.sorted_route, rb.sorted_route)
    assert torch.equal(ra.y.view(torch.int32), rb.y.view(torch.int32))


def test_unknown_chain_implementation_is_rejected(rrlib, cuda):
    from raggedroute_b200._lib import RaggedRouteError
    t, k, e, n = 16, 8, 4, 8
    buf = rrlib.ChainBuffers.allocate(t, k, e, n, cuda)
    x = torch.zeros(t, k, device=cuda)
    with pytest.raises(RaggedRouteError):
        rrlib.chain_from_tokens(x, torch.zeros(k, e, device=cuda), torch.zeros(e, k, n, device=cuda),
                                buf, ctx=rrlib.Context(implementation_id=7))
