"""The allocation-free token_permute entry point (rr_token_permute_no_alloc).

It serves callers that cannot allocate device memory: engines whose memory
planner owns every device byte, and bindings that can pass existing buffers
but cannot reach a CUDA allocator. Its scratch is a fixed 4 KB array inside
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


# (tokens, experts, hidden): one CTA chunk, two multi-chunk cases, and a
# large input at the largest expert count, whose scratch (1024 cursors) fills
# the whole 4 KB array.
LARGE_TOKENS = 2_095_104


@pytest.mark.parametrize("tokens,experts,hidden", [(32, 8, 12), (3000, 64, 128),
                                                   (50_000, 256, 32), (LARGE_TOKENS, 1024, 4)])
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


def test_no_alloc_scratch_bound(rrlib, cuda):
    """The scratch need is the E cursors at every token count, so every
    accepted shape fits the 4 KB array; an expert count above the maximum
    is rejected before any launch."""
    lib = rrlib.lib()
    for tokens in (1, 1000, LARGE_TOKENS, 1 << 24):
        for experts in (8, 1024):
            assert rrlib.token_permute_workspace_size(tokens, experts, 2, 0) == 4 * experts
    p = ctypes.c_void_p(16)
    st = lib.rr_token_permute_no_alloc(None, p, p, None, p, None, 100, 1025, 2, 0, _ctx())
    assert st.code == rrlib.StatusCode.INVALID_ARGUMENT


def test_no_alloc_dispatch_checks_match(rrlib, cuda):
    """The dispatch checks of rr_token_permute run before the empty-call
    return: an unknown kernel variant or a non-sm_100 architecture is
    rejected with the same code by both entry points, also for T=0."""
    from raggedroute_b200._lib import RRContext
    lib = rrlib.lib()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    cases = [(rrlib.ARCH_AUTO, rrlib.FAMILY_CUDA_OPTIMIZED, 11),  # id above the accepted 1..10
             (rrlib.ARCH_AUTO, rrlib.FAMILY_CUDA_NAIVE, 1),
             (rrlib.ARCH_SM86, rrlib.FAMILY_AUTO, 0)]
    p = ctypes.c_void_p(16)
    for arch, family, impl in cases:
        for tokens in (0, 4):
            ctx = ctypes.pointer(RRContext(stream, None, 0, arch, family, impl))
            a = lib.rr_token_permute(None, p, p, None, p, None, tokens, 8, 2, 0, ctx)
            b = lib.rr_token_permute_no_alloc(None, p, p, None, p, None, tokens, 8, 2, 0, ctx)
            assert a.code != 0 and a.code == b.code, (arch, family, impl, tokens, a.code, b.code)


def test_no_alloc_after_device_reset():
    """The array's address belongs to a CUDA context. A torch-free child
    process calls both entry points, resets the device (cudaDeviceReset
    through another CUDA runtime, which destroys the primary context), checks
    that the new context has a new id, and calls both again on fresh
    buffers: the no-alloc results must still equal rr_token_permute's and the
    numpy stable permute, bit for bit."""
    import os
    import subprocess
    import sys
    worker = os.path.join(os.path.dirname(os.path.abspath(__file__)), "no_alloc_reset_worker.py")
    env = dict(os.environ)
    env.setdefault("CUDA_VISIBLE_DEVICES", "0")
    res = subprocess.run([sys.executable, worker], capture_output=True, text=True, timeout=300,
                         env=env)
    assert res.returncode == 0, res.stdout + res.stderr
    assert "OK" in res.stdout, res.stdout
