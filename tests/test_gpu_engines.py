"""Engine selection of the tcgen05 GEMMs, run in child processes because the
selection is read once per process:

* the grouped GEMM on the CTA-pair engine with the 3xTF32 split
  (RAGGEDROUTE_B200_GEMM_MIXED=0) and on the one-CTA engine
  (RAGGEDROUTE_B200_GEMM_PAIRS=0) gives the same output bit for bit (same
  split, same K order, same promotion), and so does the row-gathering GEMM
  (one-CTA engine, 3xTF32) in every setting;
* the default pair engine (mixed split: TF32 hi.hi plus bfloat16 correction
  products, at K >= 128) and both 3xTF32 engines hold the FP32 contract
  against FP64 (accumulation-aware bound and 1e-5 normwise) on sampled rows;
* the router-shape dense GEMM (N = 128, rows for two waves) through the
  transposed narrow kernel (default) and through the engine
  (RAGGEDROUTE_B200_NARROW_DENSE=0) both hold the FP32 contract against FP64
  (accumulation-aware bound and 1e-5 normwise); they are not bit-identical.
"""
from __future__ import annotations

import os
import subprocess
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(tmp_path, name, env_extra):
    out = tmp_path / f"{name}.npz"
    env = dict(os.environ, **env_extra)
    res = subprocess.run([sys.executable, os.path.join(ROOT, "tests", "engine_worker.py"),
                          str(out)], capture_output=True, text=True, env=env, cwd=ROOT,
                         timeout=600)
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-2000:]
    return np.load(out)


def test_engines_agree(rrlib, oracle, cuda, tmp_path):
    default = _run(tmp_path, "default", {})
    tf32 = _run(tmp_path, "tf32", {"RAGGEDROUTE_B200_GEMM_MIXED": "0"})
    single = _run(tmp_path, "single", {"RAGGEDROUTE_B200_GEMM_PAIRS": "0",
                                       "RAGGEDROUTE_B200_NARROW_DENSE": "0"})
    assert not np.isnan(default["y"]).any()
    assert np.array_equal(tf32["y"].view(np.int32), single["y"].view(np.int32))
    for run in (default, tf32, single):
        assert np.array_equal(run["y_gather"].view(np.int32), tf32["y"].view(np.int32))
    offsets, rows = default["offsets"], default["y_rows"]
    expert = np.searchsorted(offsets, rows, side="right") - 1
    xr, w = default["x_rows"], default["w"]
    ref = np.einsum("rk,rkn->rn", xr.astype(np.float64), w[expert].astype(np.float64))
    for run in (default, tf32):
        got = run["y"][rows]
        for i, e in enumerate(expert):
            b = oracle.gemm_error_bound(xr[i:i + 1], w[e], xr.shape[1])
            assert np.all(np.abs(got[i:i + 1].astype(np.float64) - ref[i:i + 1]) <= b), (i, e)
        assert oracle.normwise_rel_error(got, ref) <= 1e-5
    a, b = default["a_rows"], default["b"]
    ref = oracle.dense_gemm_f64(a, b)
    bound = oracle.gemm_error_bound(a, b, a.shape[1])
    for run in (default, single):
        c = run["c_rows"]
        assert np.all(np.abs(c.astype(np.float64) - ref) <= bound)
        assert oracle.normwise_rel_error(c, ref) <= 1e-5
