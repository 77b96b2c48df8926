"""rr_chain_from_tokens_host: the chunked, copy-overlapped chain over host
memory must give the same Y (and routing decisions) bit for bit as
rr_chain_from_tokens over the whole batch on the device: several chunks with
a ragged last one, a batch smaller than one
chunk, an empty batch, pageable host memory, a batch of 40000 tokens in
chunks of 8192 (the whole batch and its chunks on either side of two waves
of router tiles), and a plan reused across calls (with and without the
input-ready flag that lets back-to-back calls overlap)."""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

K, E, N = 256, 64, 192


def _weights(dev):
    from raggedroute_b200.workloads import normal, zipf_log_bias
    wr = normal((K, E), 1 / 16, 21, dev)
    we = normal((E, K, N), 1 / 16, 22, dev)
    bias = torch.from_numpy(zipf_log_bias(E, 1.0)).to(dev)
    return wr, we, bias


def _device_chain(rrlib, x_host, wr, we, bias, dev):
    t = x_host.shape[0]
    buf = rrlib.ChainBuffers.allocate(t, K, E, N, dev)
    rrlib.chain_from_tokens(x_host.to(dev), wr, we, buf, logit_bias=bias)
    torch.cuda.synchronize()
    return buf


@pytest.mark.parametrize("tokens,chunk,pinned", [(5000, 1024, True), (300, 1024, True),
                                                 (4096, 1024, False), (0, 512, True),
                                                 (40000, 8192, True)])
def test_host_chain_matches_device_chain(rrlib, cuda, tokens, chunk, pinned):
    from raggedroute_b200.workloads import normal
    wr, we, bias = _weights(cuda)
    x = normal((tokens, K), 1.0, 23, "cpu")
    y = torch.full((tokens, N), float("nan"))
    ids = torch.full((tokens, 2), -1, dtype=torch.int32)
    w = torch.full((tokens, 2), float("nan"))
    if pinned:
        x, y, ids, w = x.pin_memory(), y.pin_memory(), ids.pin_memory(), w.pin_memory()
    hc = rrlib.HostChain(chunk, K, E, N)
    hc(x, wr, we, y, logit_bias=bias, expert_ids_host=ids, route_weights_host=w)
    torch.cuda.synchronize()
    hc.close()
    if tokens == 0:
        return
    ref = _device_chain(rrlib, x, wr, we, bias, cuda)
    assert torch.equal(ids, ref.expert_ids.cpu())
    assert torch.equal(w, ref.route_weights.cpu())
    assert torch.equal(y.view(torch.int32), ref.y.cpu().view(torch.int32))


@pytest.mark.parametrize("input_ready", [False, True])
def test_host_chain_plan_reused_across_calls(rrlib, cuda, input_ready):
    """Calls queued back to back; with input_ready the copies of a call may
    start while the previous call still computes (RR_HOST_CHAIN_INPUT_READY)."""
    from raggedroute_b200.workloads import normal
    wr, we, bias = _weights(cuda)
    hc = rrlib.HostChain(700, K, E, N, input_ready=input_ready)
    xs = [normal((2100 + 333 * i, K), 1.0, 30 + i, "cpu").pin_memory() for i in range(3)]
    ys = [torch.empty(x.shape[0], N).pin_memory() for x in xs]
    stream = torch.cuda.Stream(cuda)
    ctx = rrlib.Context(stream=stream.cuda_stream)
    for x, y in zip(xs, ys):
        hc(x, wr, we, y, logit_bias=bias, ctx=ctx)  # queued back to back
    stream.synchronize()
    for x, y in zip(xs, ys):
        ref = _device_chain(rrlib, x, wr, we, bias, cuda)
        assert torch.equal(y.view(torch.int32), ref.y.cpu().view(torch.int32))
    hc.close()
