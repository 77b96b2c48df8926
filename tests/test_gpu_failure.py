"""Failure detection on the GPU without a GPU fault: a bounded mbarrier wait
(the GEMM's own wait code) on a barrier that nothing arrives on gives up
after its limit, records the timeout bit in the device error word, and
returns; the context stays usable (a GEMM right after is exact)."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _consume(rrlib) -> int:
    w = ctypes.c_uint32(0)
    st = rrlib.lib().rr_consume_device_error(
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), ctypes.byref(w))
    assert st.code == 0
    return int(w.value)


def test_bounded_wait_times_out_and_reports(rrlib, oracle, cuda):
    _consume(rrlib)  # start clean
    elapsed = torch.zeros(1, dtype=torch.int64, device=cuda)
    limit = 50_000_000  # 50 ms
    st = rrlib.lib().rr_bounded_wait_selftest(
        limit, ctypes.c_void_p(elapsed.data_ptr()),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st.code == 0
    word = _consume(rrlib)
    assert word & 1, word  # kErrMbarTimeout
    waited = int(elapsed.item())
    assert limit <= waited < 20 * limit, waited
    # The context is still healthy: an exact tcgen05 GEMM right after.
    rng = np.random.default_rng(0)
    a = rng.uniform(-1, 1, (256, 64)).astype(np.float32)
    b = rng.normal(0, 0.1, (64, 96)).astype(np.float32)
    c = torch.empty(256, 96, device=cuda)
    rrlib.dense_gemm(torch.from_numpy(a).to(cuda), torch.from_numpy(b).to(cuda), c, 256, 96, 64)
    torch.cuda.synchronize()
    ref = oracle.dense_gemm_f64(a, b)
    assert oracle.normwise_rel_error(c.cpu().numpy(), ref) <= 1e-5
    assert _consume(rrlib) == 0
