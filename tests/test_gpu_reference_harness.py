"""The reference's own acceptance tests, built against this library by
tests/reference_harness/build_harness.py (from the reference sources, in the
build container) and run here on the B200:

* correctness_framework_tests (unchanged): the naive-launcher contracts,
  the correctness framework's self-tests and its randomized reference suite
  (suites selftest, edge, stream, randomized). Its `dtype` suite is not
  run: it asserts the capability levels the reference's own framework
  assigns on SM86 (FP8/FP6/FP4 "reference-only"), which B200 runs natively;
  it exercises no code of this library;
* operator_api_tests (two adaptations: SM100 instead of SM86 as the executed
  architecture, and 1024 instead of 64 as the expert cap the scan enforces):
  dispatch, argument/workspace contracts, and every operator through the
  public API with guarded buffers;
* chain_harness: the reference's registry and adapters running every L3
  chain variant, every operator variant and the CUDA-graph replays on this
  library. Variants of the reference's SM86 research study whose launchers
  this library does not implement report UNSUPPORTED; every chain variant
  the reference's L3 runs through the public API or the candidate launchers
  must PASS.
"""
from __future__ import annotations

import os
import re
import subprocess

import pytest

pytestmark = pytest.mark.gpu

BIN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "reference_harness", "_bin")

# Chain variants that run entirely through the public API and the candidate
# launchers (benchmarks/adapters/chain_adapter.cpp:263-467): all must pass.
REQUIRED_CHAINS = {
    "chain_from_tokens": ["cuda_naive", "cuda_permute_candidate", "cuda_grouped_sm86_fp32_v1",
                          "cuda_unpermute_candidate", "cuda_fused_histogram_scan",
                          "cuda_all_candidates_chain"],
    "chain_from_logits": ["cuda_naive", "cuda_permute_candidate", "cuda_grouped_sm86_fp32_v1",
                          "cuda_unpermute_candidate", "cuda_fused_histogram_scan",
                          "cuda_postlogit_retained_main", "cuda_postlogit_integrated_latest",
                          "cuda_postlogit_research_v3", "cuda_postlogit_grouped_v10"],
}


def _run(name: str, *args: str, timeout: int = 600) -> subprocess.CompletedProcess:
    path = os.path.join(BIN, name)
    assert os.path.exists(path), (
        f"{path} is missing: build it with python tests/reference_harness/build_harness.py "
        "in a checkout that has the reference sources")
    return subprocess.run([path, *args], capture_output=True, text=True, timeout=timeout)


@pytest.mark.parametrize("suite", ["selftest", "edge", "stream", "randomized"])
def test_reference_correctness_framework_tests(rrlib, cuda, suite):
    res = _run("correctness_framework_tests", "--suite", suite)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
    assert f"PASS correctness framework suite={suite}" in res.stdout


def test_reference_operator_api_tests(rrlib, cuda):
    res = _run("operator_api_tests")
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
    assert "PASS operator API tests" in res.stdout


def test_reference_chain_harness(rrlib, cuda):
    res = _run("chain_harness", timeout=900)
    out = res.stdout
    assert res.returncode == 0, out[-6000:] + res.stderr[-3000:]
    assert re.search(r"SUMMARY pass=\d+ unsupported=\d+ fail=0", out), out[-2000:]
    passed = set(re.findall(r"^PASS (\S+)", out, re.M))
    for suite, variants in REQUIRED_CHAINS.items():
        for v in variants:
            assert f"{suite}/{v}" in passed, f"{suite}/{v} did not pass"
    # every operator's cuda_naive cases, and the graph replays
    for op in ("dense_gemm", "topk_gate", "histogram", "exclusive_scan", "token_permute",
               "grouped_gemm", "unpermute"):
        assert f"{op}/cuda_naive" in passed, op
    for v in ("graph_fixed_v1", "graph_param_update_v2", "graph_exec_update_v3",
              "graph_cache_v4"):
        assert f"chain_from_logits/cuda_postlogit_{v}" in passed, v
    assert "chain_from_route_ids/cuda_postroute_current_v1" in passed
