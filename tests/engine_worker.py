"""Child process of tests/test_gpu_engines.py: runs a ragged grouped GEMM and a
router-shape dense GEMM with the engine selection the environment sets
(RAGGEDROUTE_B200_GEMM_PAIRS, RAGGEDROUTE_B200_GEMM_MIXED,
RAGGEDROUTE_B200_NARROW_DENSE) and saves the
outputs to the .npz path given as argv[1]. Inputs are seeded, so two runs
with different settings see the same data."""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main() -> int:
    import raggedroute_b200 as rr
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(21)
    sizes = rng.integers(0, 2400, 16).astype(np.int32)
    sizes[[3, 9]] = 0
    offsets = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int32)
    r, e, k, n = int(offsets[-1]), 16, 1024, 384
    g = torch.Generator(device=dev)
    g.manual_seed(21)
    x = torch.randn(r, k, generator=g, device=dev)
    w = torch.randn(e, k, n, generator=g, device=dev) / 32.0
    y = torch.full((r, n), float("nan"), device=dev)
    offsets_t = torch.from_numpy(offsets).to(dev)
    rr.grouped_gemm(x, w, offsets_t, y, e, k, n, r)
    # The row-gathering GEMM (one-CTA engine, 3xTF32) with the identity row
    # map: row r reads x[r].
    y_gather = torch.full((r, n), float("nan"), device=dev)
    rr.grouped_gemm_gather(x, torch.arange(r, dtype=torch.int32, device=dev), 1, w, offsets_t,
                           y_gather, r)
    m, kd, nd = 40000, 512, 128
    a = torch.randn(m, kd, generator=g, device=dev)
    b = torch.randn(kd, nd, generator=g, device=dev) / 16.0
    c = torch.full((m, nd), float("nan"), device=dev)
    rr.dense_gemm(a, b, c, m, nd, kd)
    torch.cuda.synchronize()
    rows = np.arange(0, m, 37)
    yrows = np.arange(0, r, 29)
    np.savez(sys.argv[1], y=y.cpu().numpy(), y_gather=y_gather.cpu().numpy(), offsets=offsets, c_rows=c.cpu().numpy()[rows],
             a_rows=a.cpu().numpy()[rows], b=b.cpu().numpy(), y_rows=yrows,
             x_rows=x.cpu().numpy()[yrows], w=w.cpu().numpy())
    print("ok")
    return 0


if __name__ == "__main__":
    sys.exit(main())
