"""Redzone canaries around every device buffer, after every call.

The reference's harness wraps each device buffer in 256-byte canary zones of
0xA5 with 0xCD poison in the output body (include/raggedroute/correctness/
guarded_buffer.h:229-316) and checks the canaries after each call
(tests/operator_api_tests.cpp). Here every input, output and workspace of
each operator and chain is carved out of its own guarded allocation; after the
call all canaries must be intact. Shapes are ragged (K, N not multiples of the
tile sizes; one case with K not a multiple of 4, which takes the FP32 path),
and the operator-by-operator pipeline must give the chain's outputs bit for
bit.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

GUARD = 256
CANARY = 0xA5
POISON = 0xCD


class Arena:
    """Guarded device buffers: [GUARD canary | body | GUARD canary]."""

    def __init__(self, device):
        self.device = device
        self.zones = []

    def out(self, shape, dtype):
        """A buffer whose body starts as 0xCD poison."""
        return self._carve(shape, dtype, None)

    def inp(self, value: torch.Tensor):
        """A buffer holding a copy of `value`."""
        return self._carve(tuple(value.shape), value.dtype, value)

    def _carve(self, shape, dtype, value):
        itemsize = torch.empty((), dtype=dtype).element_size()
        nbytes = int(np.prod(shape)) * itemsize if len(shape) else itemsize
        raw = torch.full((GUARD + ((nbytes + 15) // 16) * 16 + GUARD,), CANARY, dtype=torch.uint8,
                         device=self.device)
        body = raw[GUARD:GUARD + nbytes]
        body.fill_(POISON)
        t = body.view(dtype).view(shape)
        if value is not None:
            t.copy_(value.to(self.device))
        self.zones.append((raw, nbytes))
        return t

    def check(self, what: str):
        torch.cuda.synchronize()
        for i, (raw, nbytes) in enumerate(self.zones):
            head = raw[:GUARD]
            tail = raw[GUARD + nbytes:]
            assert bool((head == CANARY).all()), f"{what}: zone {i} leading canary overwritten"
            assert bool((tail == CANARY).all()), f"{what}: zone {i} trailing canary overwritten"


def _problem(t, k, e, n, seed):
    from raggedroute_b200.workloads import normal, uniform, zipf_log_bias
    x = uniform((t, k), seed, "cpu")
    wr = normal((k, e), 1 / np.sqrt(k), seed + 1, "cpu")
    we = normal((e, k, n), 1 / np.sqrt(k), seed + 2, "cpu")
    bias = torch.from_numpy(zipf_log_bias(e, 1.0)).float()
    return x, wr, we, bias


@pytest.mark.parametrize("t,k,e,n", [(1000, 260, 37, 100), (513, 258, 64, 130),
                                     (3000, 512, 128, 1408)])
def test_operators_and_chains_stay_inside_their_buffers(rrlib, cuda, t, k, e, n):
    a = Arena(cuda)
    x_c, wr_c, we_c, bias_c = _problem(t, k, e, n, seed=t + k)
    x, wr, we, bias = a.inp(x_c), a.inp(wr_c), a.inp(we_c), a.inp(bias_c)
    r = 2 * t
    logits = a.out((t, e), torch.float32)
    rrlib.dense_gemm(x, wr, logits, t, e, k)
    a.check("dense_gemm")
    ids = a.out((t, 2), torch.int32)
    w = a.out((t, 2), torch.float32)
    rrlib.topk_gate_biased(logits, bias, ids, w, t, e)
    a.check("topk_gate")
    counts = a.out((e,), torch.int32)
    offsets = a.out((e + 1,), torch.int32)
    rrlib.histogram(ids, counts, r, e)
    a.check("histogram")
    rrlib.exclusive_scan(counts, offsets, e)
    a.check("exclusive_scan")
    counts2 = a.out((e,), torch.int32)
    offsets2 = a.out((e + 1,), torch.int32)
    rrlib.histogram_exclusive_scan(ids, counts2, offsets2, r, e)
    a.check("histogram_exclusive_scan")
    assert torch.equal(offsets, offsets2) and torch.equal(counts, counts2)
    ws = a.out((max(1, rrlib.token_permute_workspace_size(t, e, 2, k)),), torch.uint8)
    xp = a.out((r, k), torch.float32)
    pos = a.out((r,), torch.int32)
    srt = a.out((r,), torch.int32)
    rrlib.token_permute(x, ids, offsets, xp, pos, srt, t, e, 2, k, ws)
    a.check("token_permute")
    yp = a.out((r, n), torch.float32)
    rrlib.grouped_gemm(xp, we, offsets, yp, e, k, n, r)
    a.check("grouped_gemm")
    y = a.out((t, n), torch.float32)
    rrlib.unpermute(yp, pos, w, y, t, 2, n)
    a.check("unpermute")

    # The chains, every buffer guarded; outputs equal the step-by-step ones.
    for name in ("tokens", "logits"):
        buf = rrlib.ChainBuffers(
            logits=a.out((t, e), torch.float32),
            expert_ids=a.out((t, 2), torch.int32),
            route_weights=a.out((t, 2), torch.float32),
            counts=a.out((e,), torch.int32),
            offsets=a.out((e + 1,), torch.int32),
            x_permuted=a.out((r, k), torch.float32),
            route_pos=a.out((r,), torch.int32),
            y_permuted=a.out((r, n), torch.float32),
            y=a.out((t, n), torch.float32),
            workspace=a.out((max(1, rrlib.chain_workspace_size(t, k, e, n)),), torch.uint8))
        if name == "tokens":
            rrlib.chain_from_tokens(x, wr, we, buf, logit_bias=bias)
            a.check("chain_from_tokens")
            assert torch.equal(buf.logits.view(torch.int32), logits.view(torch.int32))
        else:
            biased = a.inp(logits + bias)
            rrlib.chain_from_logits(biased, x, we, buf)
            a.check("chain_from_logits")
        assert torch.equal(buf.expert_ids, ids)
        assert torch.equal(buf.route_weights.view(torch.int32), w.view(torch.int32))
        assert torch.equal(buf.route_pos, pos)
        assert torch.equal(buf.y.view(torch.int32), y.view(torch.int32))


@pytest.mark.parametrize("top_k", [1, 4, 8])
def test_route_chain_stays_inside_its_buffers(rrlib, cuda, top_k):
    from route_ids import make_route_ids, make_route_weights
    t, k, e, n = 700, 132, 40, 68
    a = Arena(cuda)
    x_c, _, we_c, _ = _problem(t, k, e, n, seed=top_k)
    x, we = a.inp(x_c), a.inp(we_c)
    ids = a.inp(torch.from_numpy(make_route_ids(t, top_k, e, "zipf", seed=top_k)))
    rw = a.inp(torch.from_numpy(make_route_weights(t, top_k, seed=top_k)))
    r = t * top_k
    buf = rrlib.RouteChainBuffers(
        counts=a.out((e,), torch.int32), offsets=a.out((e + 1,), torch.int32),
        x_permuted=a.out((r, k), torch.float32), route_pos=a.out((r,), torch.int32),
        sorted_route=a.out((r,), torch.int32), y_permuted=a.out((r, n), torch.float32),
        y=a.out((t, n), torch.float32),
        workspace=a.out((max(1, int(rrlib.lib().rr_route_chain_workspace_size(t, top_k, e))),),
                        torch.uint8))
    rrlib.chain_from_route_ids(x, ids, rw, we, buf)
    a.check(f"chain_from_route_ids top_k={top_k}")
    assert int(buf.offsets[-1]) == r
