"""CUDA-graph capture of chains (rr_graph_*): a captured chain_from_tokens
replayed after new tokens are written into its input buffer gives the same
output, ids and positions bit for bit as a direct call on those tokens
(C1 shapes, and a second routing that changes every expert's row count);
the same for chain_from_route_ids; capture on the legacy default stream is
refused."""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_graph_chain_from_tokens_replays_new_routing(rrlib, cuda):
    from raggedroute_b200.workloads import normal, zipf_log_bias
    t, k, e, n = 512, 256, 32, 64  # C1
    x = normal((t, k), 1.0, 1, cuda)
    wr = normal((k, e), 1 / 16, 2, cuda)
    we = normal((e, k, n), 1 / 16, 3, cuda)
    bias = torch.from_numpy(zipf_log_bias(e, 1.0)).to(cuda)
    buf = rrlib.ChainBuffers.allocate(t, k, e, n, cuda)
    ref = rrlib.ChainBuffers.allocate(t, k, e, n, cuda)
    s = torch.cuda.Stream(cuda)
    g = rrlib.Graph.capture(
        lambda ctx: rrlib.chain_from_tokens(x, wr, we, buf, logit_bias=bias, ctx=ctx), s)
    assert g.nodes >= 7
    for seed in (10, 11, 12):
        new = normal((t, k), 1.0 + 0.5 * (seed - 10), seed, cuda)
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            x.copy_(new)
        g.launch(s)
        s.synchronize()
        rrlib.chain_from_tokens(new, wr, we, ref, logit_bias=bias)
        torch.cuda.synchronize()
        assert torch.equal(buf.expert_ids, ref.expert_ids)
        assert torch.equal(buf.counts, ref.counts)
        assert torch.equal(buf.route_pos, ref.route_pos)
        assert torch.equal(buf.y.view(torch.int32), ref.y.view(torch.int32))
    g.close()


def test_graph_chain_from_route_ids(rrlib, cuda):
    from route_ids import make_route_ids, make_route_weights
    t, k, e, n, top_k = 257, 128, 16, 96, 4
    rng = np.random.default_rng(7)
    x = torch.from_numpy(rng.uniform(-1, 1, (t, k)).astype(np.float32)).to(cuda)
    w = torch.from_numpy(rng.normal(0, 0.1, (e, k, n)).astype(np.float32)).to(cuda)
    ids = torch.zeros(t, top_k, dtype=torch.int32, device=cuda)
    rw = torch.zeros(t, top_k, device=cuda)
    buf = rrlib.RouteChainBuffers.allocate(t, top_k, k, e, n, cuda)
    ref = rrlib.RouteChainBuffers.allocate(t, top_k, k, e, n, cuda)
    s = torch.cuda.Stream(cuda)
    g = rrlib.Graph.capture(lambda ctx: rrlib.chain_from_route_ids(x, ids, rw, w, buf, ctx=ctx), s)
    for seed, dist in ((1, "zipf"), (2, "uniform"), (3, "duplicate_route")):
        new_ids = torch.from_numpy(make_route_ids(t, top_k, e, dist, 1.3, seed)).to(cuda)
        new_w = torch.from_numpy(make_route_weights(t, top_k, seed)).to(cuda)
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            ids.copy_(new_ids)
            rw.copy_(new_w)
        g.launch(s)
        s.synchronize()
        rrlib.chain_from_route_ids(x, new_ids, new_w, w, ref)
        torch.cuda.synchronize()
        assert torch.equal(buf.counts, ref.counts)
        assert torch.equal(buf.sorted_route, ref.sorted_route)
        assert torch.equal(buf.y.view(torch.int32), ref.y.view(torch.int32))
    g.close()


def test_graph_capture_refuses_default_stream(rrlib, cuda):
    from raggedroute_b200._lib import RaggedRouteError, check
    with pytest.raises(RaggedRouteError):
        check(rrlib.lib().rr_graph_capture_begin(None), "rr_graph_capture_begin")
