"""ops::launch_cache_scrub (src/benchmark/cache_scrub.cu:17-50): every word
of the buffer is rewritten in place as v * 1664525 + 1013904223 + index
(mod 2^32), words past the given count stay untouched, zero elements is a
no-op returning success, and a null buffer with work is rejected with
cudaErrorInvalidValue (1). Counts cover one partial block, an odd count above
one grid-stride pass of the launch, and a 256 MiB buffer (the bench's scrub
size, twice the L2)."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def expected(before: np.ndarray) -> np.ndarray:
    idx = np.arange(before.size, dtype=np.uint64)
    v = before.astype(np.uint64) * np.uint64(1664525) + np.uint64(1013904223) + idx
    return (v & np.uint64(0xFFFFFFFF)).astype(np.uint32)


def scrub(rrlib, buf: torch.Tensor, elements: int) -> int:
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    return rrlib.lib().rr_launch_cache_scrub(ctypes.c_void_p(buf.data_ptr()), elements, stream)


@pytest.mark.parametrize("elements", [1, 255, 1_000_003, 64 << 20])
def test_cache_scrub_rewrites_every_word(rrlib, cuda, elements):
    rng = np.random.default_rng(elements)
    before = rng.integers(0, 2**32, elements + 64, dtype=np.uint64).astype(np.uint32)
    buf = torch.from_numpy(before.view(np.int32)).to(cuda)
    assert scrub(rrlib, buf, elements) == 0
    torch.cuda.synchronize()
    after = buf.cpu().numpy().view(np.uint32)
    assert np.array_equal(after[:elements], expected(before[:elements]))
    assert np.array_equal(after[elements:], before[elements:])
    # A second pass applies the same map to the new contents.
    assert scrub(rrlib, buf, elements) == 0
    torch.cuda.synchronize()
    again = buf.cpu().numpy().view(np.uint32)
    assert np.array_equal(again[:elements], expected(after[:elements]))


def test_cache_scrub_empty_and_null(rrlib, cuda):
    buf = torch.arange(16, dtype=torch.int32, device=cuda)
    assert scrub(rrlib, buf, 0) == 0
    torch.cuda.synchronize()
    assert torch.equal(buf, torch.arange(16, dtype=torch.int32, device=cuda))
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert rrlib.lib().rr_launch_cache_scrub(None, 0, stream) == 0
    assert rrlib.lib().rr_launch_cache_scrub(None, 8, stream) == 1  # cudaErrorInvalidValue
