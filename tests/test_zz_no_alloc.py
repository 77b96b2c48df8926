"""The allocation-free token_permute entry point (rr_token_permute_no_alloc).

It serves callers that cannot allocate device memory: engines whose memory
planner owns every device byte, and bindings that can pass existing buffers
but cannot reach a CUDA allocator. Its scratch is a fixed 4 MiB array inside
the library. These tests call it through the C ABI and require results
identical to rr_token_permute (bit-exact: routing metadata and row copies
are integer/byte work) on two calls in a row, so a second call that reuses
the array's leftover contents is covered. The file sorts last so that a run
stopping at the first failure has already run every other test.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ctx():
    from raggedroute_b200._lib import RRContext
    return ctypes.pointer(RRContext(ctypes.c_void_p(torch.cuda.current_stream().cuda_stream),
                                    None, 0, 0, 0, 0))


@pytest.mark.parametrize("tokens,experts,hidden", [(3000, 64, 128), (50_000, 256, 32)])
def test_no_alloc_matches_workspace_permute(rrlib, cuda, tokens, experts, hidden):
    lib = rrlib.lib()
    rng = np.random.default_rng(tokens + experts)
    top_k = 2
    routes = tokens * top_k
    x = torch.rand(tokens, hidden, device=cuda)
    for call in range(2):
        ids_np = rng.integers(0, experts, routes).astype(np.int32)
        counts = np.bincount(ids_np, minlength=experts)
        offsets_np = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
        ids = torch.from_numpy(ids_np).to(cuda)
        offsets = torch.from_numpy(offsets_np).to(cuda)
        xp_ref = torch.empty(routes, hidden, device=cuda)
        pos_ref = torch.empty(routes, dtype=torch.int32, device=cuda)
        sr_ref = torch.empty(routes, dtype=torch.int32, device=cuda)
        ws_bytes = rrlib.token_permute_workspace_size(tokens, experts, top_k, hidden)
        ws = torch.empty(ws_bytes // 4 + 1, dtype=torch.int32, device=cuda)
        rrlib.token_permute(x, ids, offsets, xp_ref, pos_ref, sr_ref, tokens, experts, top_k,
                            hidden, ws)
        xp = torch.full((routes, hidden), float("nan"), device=cuda)
        pos = torch.full((routes,), -1, dtype=torch.int32, device=cuda)
        sr = torch.full((routes,), -1, dtype=torch.int32, device=cuda)
        st = lib.rr_token_permute_no_alloc(x.data_ptr(), ids.data_ptr(), offsets.data_ptr(),
                                           xp.data_ptr(), pos.data_ptr(), sr.data_ptr(), tokens,
                                           experts, top_k, hidden, _ctx())
        assert st.code == 0, st.message
        torch.cuda.synchronize()
        assert torch.equal(pos, pos_ref), f"call {call}: route_pos differs"
        assert torch.equal(sr, sr_ref), f"call {call}: sorted_route differs"
        assert torch.equal(xp.view(torch.int32), xp_ref.view(torch.int32)), f"call {call}: rows"


def test_no_alloc_rejects_oversize(rrlib, cuda):
    lib = rrlib.lib()
    tokens, experts = 1 << 24, 1024  # scratch need far above 4 MiB
    assert rrlib.token_permute_workspace_size(tokens, experts, 2, 0) > (4 << 20)
    p = ctypes.c_void_p(16)
    st = lib.rr_token_permute_no_alloc(None, p, p, None, p, None, tokens, experts, 2, 0, _ctx())
    assert st.code == rrlib.StatusCode.INVALID_ARGUMENT
    assert b"4 MiB" in st.message
