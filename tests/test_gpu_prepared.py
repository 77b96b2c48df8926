"""Prepared expert weights (rr_prepare_expert_weights, new API).

* The prepared layout itself: hi = W^T and lo = W^T - trunc_tf32(W^T),
  bit for bit.
* rr_grouped_gemm_prepared against the FP64 oracle with the same tolerances
  as the raw-weight engine (the reference's accumulation-aware bound
  elementwise and 1e-5 normwise), over ragged and empty groups, N not a
  multiple of the 256-column tile, K up to 4096.
* chain_from_tokens / chain_from_logits on prepared weights: routing is the
  raw-weight chain's bit for bit (the router GEMM is unchanged) and the
  output is within the FP32 tolerance of it and of the oracle.
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


def error_word(rrlib) -> int:
    w = ctypes.c_uint32(0)
    st = rrlib.lib().rr_consume_device_error(
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), ctypes.byref(w))
    assert st.code == 0
    return int(w.value)


def test_prepared_layout_bits(rrlib, cuda):
    e, k, n = 3, 40, 36
    w = torch.randn(e, k, n, device=cuda)
    p = rrlib.PreparedExpertWeights(w)
    torch.cuda.synchronize()
    half = int(rrlib.lib().rr_prepared_expert_weights_size(e, k, n)) // 2
    assert half % 256 == 0 and half >= e * k * n * 4
    hi = p.buffer[:e * n * k * 4].view(torch.float32).view(e, n, k)
    lo = p.buffer[half:half + e * n * k * 4].view(torch.float32).view(e, n, k)
    wt = w.transpose(1, 2).contiguous()
    assert torch.equal(hi.view(torch.int32), wt.view(torch.int32))
    trunc = (wt.view(torch.int32) & ~0x1FFF).view(torch.float32)
    assert torch.equal(lo.view(torch.int32), (wt - trunc).view(torch.int32))


@pytest.mark.parametrize("sizes,k,n", [
    ([128], 16, 256),
    ([1, 0, 0, 5, 127, 129, 0, 300], 64, 100),
    ([0, 0, 17], 40, 1408),
    ([2000, 7, 0, 513], 512, 384),
    ([64] * 16, 4096, 128),
    ([900, 1100, 333], 4096, 1408),
])
def test_grouped_gemm_prepared_accuracy(rrlib, oracle, cuda, sizes, k, n):
    rng = np.random.default_rng(len(sizes) * 17 + k + n)
    sizes = np.asarray(sizes, np.int32)
    e = sizes.size
    offsets = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int32)
    r = int(offsets[-1])
    x = rng.uniform(-1, 1, (r, k)).astype(np.float32)
    w = rng.normal(0, 1 / math.sqrt(k), (e, k, n)).astype(np.float32)
    prep = rrlib.PreparedExpertWeights(dev(w, cuda))
    y = torch.full((r, n), float("nan"), device=cuda)
    rrlib.grouped_gemm_prepared(dev(x, cuda), prep, dev(offsets, cuda), y, r)
    torch.cuda.synchronize()
    got = y.cpu().numpy()
    ref = oracle.grouped_gemm_f64(x, w, offsets)
    for i in range(e):
        s = slice(offsets[i], offsets[i + 1])
        if offsets[i + 1] > offsets[i]:
            bound = oracle.gemm_error_bound(x[s], w[i], k)
            err = np.abs(got[s].astype(np.float64) - ref[s])
            assert np.all(err <= bound), float((err - bound).max())
    assert oracle.normwise_rel_error(got, ref) <= 1e-5
    assert error_word(rrlib) == 0


@pytest.mark.parametrize("mode", ["tokens", "logits"])
def test_chain_prepared_routing_and_output(rrlib, oracle, cuda, mode):
    from raggedroute_b200.workloads import normal, zipf_log_bias
    t, k, e, n = 3000, 512, 64, 384
    x = normal((t, k), 1.0, 61, cuda)
    wr = normal((k, e), 1 / math.sqrt(k), 62, cuda)
    we = normal((e, k, n), 1 / math.sqrt(k), 63, cuda)
    bias = torch.from_numpy(zipf_log_bias(e, 1.0)).to(cuda)
    prep = rrlib.PreparedExpertWeights(we)
    raw = rrlib.ChainBuffers.allocate(t, k, e, n, cuda)
    got = rrlib.ChainBuffers.allocate(t, k, e, n, cuda)
    if mode == "tokens":
        rrlib.chain_from_tokens(x, wr, we, raw, logit_bias=bias)
        rrlib.chain_from_tokens(x, wr, prep, got, logit_bias=bias)
    else:
        logits = x @ wr + bias
        rrlib.chain_from_logits(logits, x, we, raw)
        rrlib.chain_from_logits(logits, x, prep, got)
    torch.cuda.synchronize()
    for name in ("expert_ids", "counts", "offsets", "route_pos"):
        assert torch.equal(getattr(got, name), getattr(raw, name)), name
    assert torch.equal(got.route_weights.view(torch.int32), raw.route_weights.view(torch.int32))
    assert torch.equal(got.x_permuted.view(torch.int32), raw.x_permuted.view(torch.int32))
    ids = raw.expert_ids.cpu().numpy()
    w = raw.route_weights.cpu().numpy()
    y_ref = oracle.chain_output_f32(x.cpu().numpy(), we.cpu().numpy(), ids, w)
    ok, err, rel = oracle.compare_floating(got.y.cpu().numpy(), y_ref, 1e-4, 4e-5 * k)
    assert ok, (err, rel)
    assert oracle.normwise_rel_error(got.y.cpu().numpy(), raw.y.cpu().numpy()) <= 1e-5
    assert error_word(rrlib) == 0


def test_prepared_rejects_gather_rows(rrlib, cuda):
    t, k, e, n = 64, 32, 8, 16
    we = torch.randn(e, k, n, device=cuda)
    prep = rrlib.PreparedExpertWeights(we)
    buf = rrlib.ChainBuffers.allocate(t, k, e, n, cuda)
    with pytest.raises(ValueError):
        rrlib.chain_from_tokens(torch.randn(t, k, device=cuda), torch.randn(k, e, device=cuda),
                                prep, buf, gather_rows=True)
