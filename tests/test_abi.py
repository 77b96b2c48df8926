"""C ABI and C++ API contract checks that need no GPU.

* libraggedroute_b200.so loads and exports every rr_* entry point declared in
  include/raggedroute_b200.h, and every raggedroute:: function of the
  reference-compatible C++ headers.
* Argument validation that happens before any CUDA call returns the
  reference's status codes (explicit architecture, so no device query).
* A C++ program compiled against include/raggedroute/*.h links and passes the
  pure-dispatch contract (tests/cpp/api_contract.cpp).
"""
from __future__ import annotations

import ctypes
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "raggedroute_b200.h")


def declared_c_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(rr_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol(rrlib):
    lib = rrlib.lib()
    names = declared_c_symbols()
    assert len(names) >= 30
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    # The Python binding knows every declared symbol's signature.
    from raggedroute_b200._lib import SIGNATURES
    assert sorted(SIGNATURES) == names


def test_cpp_api_symbols_exported(rrlib):
    out = subprocess.run(["nm", "-D", "--defined-only", "-C", rrlib.library_path],
                         capture_output=True, text=True, check=True).stdout
    for fn in ["raggedroute::dense_gemm(", "raggedroute::topk_gate(", "raggedroute::histogram(",
               "raggedroute::exclusive_scan(", "raggedroute::histogram_exclusive_scan(",
               "raggedroute::token_permute(", "raggedroute::grouped_gemm(",
               "raggedroute::unpermute(", "raggedroute::select_kernel(",
               "raggedroute::ops::launch_token_permute_naive(",
               "raggedroute::ops::launch_cache_scrub(", "raggedroute::chain_from_tokens(",
               "raggedroute::get_token_permute_workspace_size("]:
        assert fn in out, fn
    # Every candidate launcher declared in include/raggedroute/candidate_ops.h.
    text = open(os.path.join(ROOT, "include", "raggedroute", "candidate_ops.h")).read()
    candidates = re.findall(r"cudaError_t (launch_[a-z0-9_]+)\(", text)
    assert len(candidates) == 7
    for fn in candidates:
        assert f"raggedroute::ops::{fn}(" in out, fn
    # The wrappers' internal helpers stay private, and the CUDA runtime is
    # the caller's (linked dynamically, not exported from here).
    assert "cudaMalloc" not in out
    assert "raggedroute::detail" not in out
    deps = subprocess.run(["readelf", "-d", rrlib.library_path], capture_output=True, text=True,
                          check=True).stdout
    assert "libcudart.so.12" in deps


def _ctx(arch=4, family=0, impl=0, ws=None, ws_bytes=0):
    from raggedroute_b200._lib import RRContext
    return ctypes.pointer(RRContext(None, ws, ws_bytes, arch, family, impl))


def test_host_validation_status_codes(rrlib):
    lib = rrlib.lib()
    S = rrlib.StatusCode
    assert lib.rr_topk_gate(None, None, None, -1, 8, 2, _ctx()).code == S.INVALID_ARGUMENT
    assert lib.rr_topk_gate(None, None, None, 0, 8, 2, _ctx()).code == S.SUCCESS
    assert lib.rr_topk_gate(None, None, None, 0, 8, 2, _ctx(arch=1)).code == \
        S.UNSUPPORTED_ARCHITECTURE
    assert lib.rr_topk_gate(None, None, None, 0, 8, 2, _ctx(family=0, impl=3)).code == \
        S.UNSUPPORTED_KERNEL_VARIANT
    assert lib.rr_topk_gate(None, None, None, 0, 8, 2, _ctx(family=2, impl=9)).code == \
        S.UNSUPPORTED_KERNEL_VARIANT
    assert lib.rr_dense_gemm(None, None, None, -1, 1, 1, _ctx()).code == S.INVALID_ARGUMENT
    assert lib.rr_histogram(None, None, 4, 2, _ctx()).code == S.INVALID_ARGUMENT
    assert lib.rr_exclusive_scan(None, None, 1025, _ctx()).code == S.INVALID_ARGUMENT
    p = ctypes.c_void_p(8)
    assert lib.rr_token_permute(None, p, p, None, p, None, 1, 2, 1, 0, _ctx()).code == \
        S.INSUFFICIENT_WORKSPACE
    assert lib.rr_token_permute(None, p, p, None, p, None, 1, 2, 3, 0, _ctx()).code == \
        S.INVALID_ARGUMENT
    assert lib.rr_grouped_gemm(None, None, None, None, 4, 7, 5, 0, _ctx()).code == S.SUCCESS
    assert lib.rr_unpermute(None, None, None, None, 1, 65, 4, _ctx()).code == S.INVALID_ARGUMENT
    assert lib.rr_dense_gemm(None, None, None, 1, 1, 1, None).code == S.INVALID_ARGUMENT
    assert lib.rr_classify_compute_capability(10, 0) == 4
    assert lib.rr_classify_compute_capability(9, 0) == 2


def test_workspace_queries(rrlib):
    lib = rrlib.lib()
    assert lib.rr_token_permute_workspace_size(1, 2, 1, 0) == 8
    assert lib.rr_token_permute_workspace_size(2, 2, 2, 2) == 8
    # The reference's E*4 cursor bytes (src/permute/operator.cpp:17-19) at
    # every size: the multi-CTA chunk table lives in route_pos.
    for tokens in (1 << 10, 1 << 19, 1 << 24):
        for experts in (2, 64, 256, 1024):
            assert lib.rr_token_permute_workspace_size(tokens, experts, 2, 128) == 4 * experts
    # The chain workspace: the permute workspace at 2T routes, 256-byte
    # aligned, then sorted_route [2T] for the row-gathering variant.
    perm = lib.rr_token_permute_workspace_size(65536, 128, 2, 4096)
    assert lib.rr_chain_workspace_size(65536, 4096, 128, 1408) == \
        (perm + 255) // 256 * 256 + 2 * 65536 * 4
    assert lib.rr_route_chain_workspace_size(1000, 4, 16) == \
        lib.rr_token_permute_workspace_size(1000, 16, 4, 0)
    for fn in ("rr_histogram_exclusive_scan_workspace_size", "rr_histogram_workspace_size"):
        assert getattr(lib, fn)(1 << 20, 64) == 0


def test_cpp_contract_program(rrlib, tmp_path):
    exe = tmp_path / "api_contract"
    src = os.path.join(ROOT, "tests", "cpp", "api_contract.cpp")
    libdir = os.path.dirname(rrlib.library_path)
    cmd = ["g++", "-std=c++17", "-O1", src, "-I" + os.path.join(ROOT, "include"),
           "-I/usr/local/cuda/include", "-L" + libdir, "-lraggedroute_b200",
           "-Wl,-rpath," + libdir, "-o", str(exe)]
    subprocess.run(cmd, check=True)
    res = subprocess.run([str(exe)], capture_output=True, text=True)
    assert res.returncode == 0, res.stdout + res.stderr
    assert "all checks passed" in res.stdout


def test_host_chain_flags_validation(rrlib):
    lib = rrlib.lib()
    st = lib.rr_host_chain_set_flags(None, 1)
    assert st.code == rrlib.StatusCode.INVALID_ARGUMENT


def test_prepared_weights_size_and_validation(rrlib):
    lib = rrlib.lib()
    half = (3 * 40 * 36 * 4 + 255) // 256 * 256
    assert lib.rr_prepared_expert_weights_size(3, 40, 36) == 2 * half
    assert lib.rr_prepared_expert_weights_size(0, 40, 36) == 0
    p = ctypes.c_void_p(256)
    # K not a multiple of 4, a misaligned buffer, a short buffer: rejected
    # before any device work (explicit architecture, no device query).
    st = lib.rr_prepare_expert_weights(p, 3, 42, 36, p, 1 << 20, _ctx())
    assert st.code == rrlib.StatusCode.INVALID_ARGUMENT
    st = lib.rr_prepare_expert_weights(p, 3, 40, 36, ctypes.c_void_p(258), 1 << 20, _ctx())
    assert st.code == rrlib.StatusCode.INVALID_ARGUMENT
    st = lib.rr_prepare_expert_weights(p, 3, 40, 36, p, 16, _ctx())
    assert st.code == rrlib.StatusCode.INSUFFICIENT_WORKSPACE
    st = lib.rr_grouped_gemm_prepared(p, p, p, p, 3, 42, 36, 10, _ctx())
    assert st.code == rrlib.StatusCode.INVALID_ARGUMENT
    # Prepared weights are a token/logit chain option only.
    from raggedroute_b200._lib import RRContext
    ctx = ctypes.pointer(RRContext(None, None, 0, 4, 0, 2))
    st = lib.rr_chain_from_route_ids(None, None, None, None, None, None, None, None, None, None,
                                     None, 1, 2, 8, 4, 8, ctx)
    assert st.code == rrlib.StatusCode.UNSUPPORTED_KERNEL_VARIANT
