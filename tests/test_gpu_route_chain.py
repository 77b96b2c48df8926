"""chain_from_route_ids (post-route chain, top_k routes per token) on the
GPU against the oracle: counts and offsets exact, route_pos and
sorted_route equal to the stable counting-sort order (hence a bijection
onto the expert segments, the reference's check,
postroute_chain_adapter.cpp:356-376), x_permuted rows bit-exact, and the
output within the reference's tolerance (atol 1e-4, rtol 4e-5*K*top_k,
postroute_chain_adapter.cpp:378) and 1e-5 normwise against the float64
composition. Shapes: the reference's own case (T=17, E=16, K=N=64,
top_k 4 and 8, every route to expert 0), every route-id distribution, and a
larger ragged case."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from route_ids import make_route_ids, make_route_weights

pytestmark = pytest.mark.gpu


def _run(rrlib, oracle, cuda, t, k, e, n, top_k, dist, zipf_s=1.4, seed=0):
    rng = np.random.default_rng(seed)
    x = rng.uniform(-1, 1, (t, k)).astype(np.float32)
    w = rng.normal(0, 1 / np.sqrt(k), (e, k, n)).astype(np.float32)
    ids = make_route_ids(t, top_k, e, dist, zipf_s, seed)
    rw = make_route_weights(t, top_k, seed)
    buf = rrlib.RouteChainBuffers.allocate(t, top_k, k, e, n, cuda)
    buf.y.fill_(float("nan"))
    rrlib.chain_from_route_ids(torch.from_numpy(x).to(cuda), torch.from_numpy(ids).to(cuda),
                               torch.from_numpy(rw).to(cuda), torch.from_numpy(w).to(cuda), buf)
    torch.cuda.synchronize()
    counts, offsets, xp, pos, sr, y = oracle.route_chain_f64(x, w, ids, rw, e)
    assert np.array_equal(buf.counts.cpu().numpy(), counts)
    assert np.array_equal(buf.offsets.cpu().numpy(), offsets)
    assert np.array_equal(buf.route_pos.cpu().numpy(), pos)
    assert np.array_equal(buf.sorted_route.cpu().numpy(), sr)
    assert np.array_equal(buf.x_permuted.cpu().numpy(), xp)
    got = buf.y.cpu().numpy()
    ok, _, _ = oracle.compare_floating(got, y.astype(np.float32), 1e-4, 4e-5 * k * top_k)
    assert ok
    assert oracle.normwise_rel_error(got, y) <= 1e-5


@pytest.mark.parametrize("top_k", [4, 8])
def test_route_chain_reference_case(rrlib, oracle, cuda, top_k):
    _run(rrlib, oracle, cuda, 17, 64, 16, 64, top_k, "duplicate_route", seed=top_k)


@pytest.mark.parametrize("dist", ["uniform", "zipf", "single_hot", "round_robin"])
@pytest.mark.parametrize("top_k", [1, 2, 4, 8])
def test_route_chain_distributions(rrlib, oracle, cuda, dist, top_k):
    _run(rrlib, oracle, cuda, 300, 128, 16, 96, top_k, dist, seed=10 * top_k + len(dist))


def test_route_chain_large_ragged(rrlib, oracle, cuda):
    _run(rrlib, oracle, cuda, 3000, 256, 64, 192, 4, "zipf", zipf_s=1.2, seed=99)


def test_route_chain_rejects_bad_top_k(rrlib, cuda):
    from raggedroute_b200._lib import RaggedRouteError
    x = torch.zeros(4, 8, device=cuda)
    w = torch.zeros(4, 8, 8, device=cuda)
    for top_k in (9, 5):  # above 8; above E=4
        ids = torch.zeros(4, top_k, dtype=torch.int32, device=cuda)
        rw = torch.zeros(4, top_k, device=cuda)
        buf = rrlib.RouteChainBuffers.allocate(4, top_k, 8, 4, 8, cuda)
        with pytest.raises(RaggedRouteError):
            rrlib.chain_from_route_ids(x, ids, rw, w, buf)


@pytest.mark.parametrize("frame", [0, 1, 2])
def test_route_trace_frames_through_both_chains(rrlib, oracle, cuda, frame):
    """A committed route-trace frame drives chain_from_logits (through the
    trace logits, chain_adapter.cpp:207-228) and chain_from_route_ids; both
    route exactly the frame's ids and match the oracle."""
    import os
    from raggedroute_b200.route_trace import load_route_trace_frame, trace_logits
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden",
                        "fixture_t24_e16_top2.rrtrace")
    fr = load_route_trace_frame(path, frame)
    t, e, k, n = fr.tokens, fr.experts, 64, 32
    rng = np.random.default_rng(frame)
    x = rng.uniform(-1, 1, (t, k)).astype(np.float32)
    w = rng.normal(0, 1 / 8, (e, k, n)).astype(np.float32)
    logits = trace_logits(fr.expert_ids, e)
    buf = rrlib.ChainBuffers.allocate(t, k, e, n, cuda)
    rrlib.chain_from_logits(torch.from_numpy(logits).to(cuda), torch.from_numpy(x).to(cuda),
                            torch.from_numpy(w).to(cuda), buf)
    torch.cuda.synchronize()
    assert np.array_equal(buf.expert_ids.cpu().numpy(), fr.expert_ids)
    ids, rw = oracle.top2_f32(logits)
    _, _, _, _, _, y = oracle.route_chain_f64(x, w, ids.reshape(-1, 2), rw.reshape(-1, 2), e)
    ok, _, _ = oracle.compare_floating(buf.y.cpu().numpy(), y.astype(np.float32), 1e-4, 4e-5 * k * 2)
    assert ok
    # The same frame as route ids, with the gate's own (device) weights.
    rbuf = rrlib.RouteChainBuffers.allocate(t, 2, k, e, n, cuda)
    rrlib.chain_from_route_ids(torch.from_numpy(x).to(cuda), torch.from_numpy(fr.expert_ids).to(cuda),
                               buf.route_weights, torch.from_numpy(w).to(cuda), rbuf)
    torch.cuda.synchronize()
    assert torch.equal(rbuf.y.view(torch.int32), buf.y.view(torch.int32))
