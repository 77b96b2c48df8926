"""Build recipe of the reference harness (TEST INFRASTRUCTURE ONLY).

Compiles RaggedRoute's own acceptance tests and benchmark adapters, from the
sources where they lie in the reference checkout, against this repository's
public headers (include/raggedroute/*.h, first on the include path) and
links them with raggedroute_b200/libraggedroute_b200.so. Nothing is copied
out of the reference: objects and binaries go to tests/reference_harness/_bin
(git-ignored; it travels with the working tree to the GPU host, which has no
reference checkout). Three programs:

* correctness_framework_tests -- tests/correctness_framework_tests.cpp,
  unchanged, with the reference's correctness framework
  (src/correctness/*, src/*/cpu_reference/*).
* operator_api_tests -- tests/operator_api_tests.cpp with the substitutions
  in OPERATOR_API_ADAPTATIONS applied to a copy under _bin (each must match
  exactly the stated number of times): the architecture the dispatch and the
  runtime tests target (SM86 in the reference, SM100 here) and the expert cap
  the scan must enforce (64 there, 1024 here). Everything else runs as
  written.
* chain_harness -- tests/reference_harness/chain_harness.cpp (this repo)
  driving the reference's benchmark registry and adapters
  (benchmarks/core/*.cpp, benchmarks/adapters/*.cpp) with
  research_stubs.cpp standing in for the SM86 research launchers this
  library does not implement.

Library baselines (cuBLAS, CUB, CUTLASS, vLLM) are configured off, as in a
reference build without those dependencies. Where the reference checkout is
(--reference, $RAGGEDROUTE_REFERENCE, else ../reference) is resolved as in
oracle/build_oracle.py.

Run: python tests/reference_harness/build_harness.py [--reference PATH] [--force]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
OUT = os.path.join(HERE, "_bin")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
CUDA_INC = "/usr/local/cuda/include"
CUDA_LIB = "/usr/local/cuda/lib64"
LIB_DIR = os.path.join(REPO, "raggedroute_b200")

# (pattern, replacement, expected count) applied to tests/operator_api_tests.cpp.
OPERATOR_API_ADAPTATIONS = [
    ('#include "../src/runtime/operator_internal.h"', '#include "runtime/operator_internal.h"', 1),
    ("request.architecture = DeviceArchitecture::kSm86;",
     "request.architecture = DeviceArchitecture::kSm100;", 3),
    ("architecture != raggedroute::DeviceArchitecture::kSm86",
     "architecture != raggedroute::DeviceArchitecture::kSm100", 1),
    ("invalid.experts = 65;", "invalid.experts = 1025;", 1),
]

CORRECTNESS_SOURCES = [
    "src/correctness/reference_validation.cpp",
    "src/correctness/report.cpp",
    "src/dense_gemm/cpu_reference/reference.cpp",
    "src/grouped_gemm/cpu_reference/reference.cpp",
    "src/histogram/cpu_reference/reference.cpp",
    "src/permute/cpu_reference/reference.cpp",
    "src/scan/cpu_reference/reference.cpp",
    "src/topk_gate/cpu_reference/reference.cpp",
    "src/unpermute/cpu_reference/reference.cpp",
]
CORRECTNESS_CUDA_SOURCES = ["src/correctness/framework.cu"]
BENCHMARK_SOURCES = ["benchmarks/core/types.cpp", "benchmarks/core/registry.cpp",
                     "benchmarks/core/runner.cpp"] + [
    f"benchmarks/adapters/{n}_adapter.cpp" for n in (
        "dense_gemm", "tensorcore_gemm", "topk_gate", "histogram", "exclusive_scan",
        "histogram_exclusive_scan", "token_permute", "grouped_gemm", "unpermute", "chain",
        "postroute_chain")]

PROGRAMS = ("correctness_framework_tests", "operator_api_tests", "chain_harness")


def reference_checkout(reference: str | None = None) -> str:
    if reference:
        return reference
    sys.path.insert(0, REPO)
    from oracle.build_oracle import reference_checkout as locate  # noqa: WPS433
    return locate()


def _flags(ref: str) -> list[str]:
    return ["-std=c++17", "-O2", "-fPIC", "-DRAGGEDROUTE_GIT_SHA=\"reference-harness\"",
            "-DRAGGEDROUTE_CUDATOOLKIT_VERSION=\"12.9\"",
            "-I" + os.path.join(REPO, "include"), "-I" + os.path.join(ref, "include"),
            "-I" + os.path.join(ref, "src"), "-I" + os.path.join(ref, "src", "dense_gemm"),
            "-I" + CUDA_INC]


def _obj_name(path: str) -> str:
    return os.path.join(OUT, "obj", path.replace(os.sep, "_").lstrip("_") + ".o")


def _compile(src: str, obj: str, flags: list[str], cuda: bool) -> str:
    if cuda:
        cmd = [NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-Xcompiler", "-fPIC"] + \
            [f for f in flags if f != "-fPIC"] + ["-c", src, "-o", obj]
    else:
        cmd = ["g++"] + flags + ["-c", src, "-o", obj]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"compile failed: {src}\n{res.stdout}\n{res.stderr}")
    return obj


def _adapted_operator_api(ref: str) -> str:
    with open(os.path.join(ref, "tests", "operator_api_tests.cpp")) as f:
        text = f.read()
    for old, new, count in OPERATOR_API_ADAPTATIONS:
        found = text.count(old)
        if found != count:
            raise RuntimeError(f"operator_api_tests.cpp: expected {count} x {old!r}, found {found}")
        text = text.replace(old, new)
    path = os.path.join(OUT, "src", "operator_api_tests_sm100.cpp")
    with open(path, "w") as f:
        f.write(text)
    return path


def _link(out: str, objs: list[str]) -> None:
    cmd = ["g++", "-o", out] + objs + [
        "-L" + LIB_DIR, "-lraggedroute_b200", "-Wl,-rpath,$ORIGIN/../../../raggedroute_b200",
        "-L" + CUDA_LIB, "-lcudart", "-Wl,-rpath," + CUDA_LIB, "-lpthread"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed: {out}\n{res.stdout}\n{res.stderr}")


def build_harness(reference: str | None = None, force: bool = False, jobs: int = 8):
    """Builds the three programs (None if the reference checkout is absent)."""
    ref = reference_checkout(reference)
    if not os.path.isdir(os.path.join(ref, "benchmarks")):
        return None
    lib = os.path.join(LIB_DIR, "libraggedroute_b200.so")
    if not os.path.exists(lib):
        raise RuntimeError(f"{lib} is missing; build the library first")
    outs = {p: os.path.join(OUT, p) for p in PROGRAMS}
    if not force and all(os.path.exists(o) and os.path.getmtime(o) >= os.path.getmtime(lib)
                         for o in outs.values()):
        return outs
    os.makedirs(os.path.join(OUT, "obj"), exist_ok=True)
    os.makedirs(os.path.join(OUT, "src"), exist_ok=True)
    flags = _flags(ref)
    jobs_list = []  # (src, obj, cuda)
    for rel in CORRECTNESS_SOURCES + BENCHMARK_SOURCES + [
            "tests/correctness_framework_tests.cpp"]:
        jobs_list.append((os.path.join(ref, rel), _obj_name(rel), False))
    for rel in CORRECTNESS_CUDA_SOURCES:
        jobs_list.append((os.path.join(ref, rel), _obj_name(rel), True))
    api_src = _adapted_operator_api(ref)
    jobs_list.append((api_src, _obj_name("operator_api_tests_sm100.cpp"), False))
    for name in ("research_stubs.cpp", "chain_harness.cpp"):
        jobs_list.append((os.path.join(HERE, name), _obj_name("harness_" + name), False))
    with cf.ThreadPoolExecutor(max_workers=max(1, jobs)) as ex:
        list(ex.map(lambda j: _compile(j[0], j[1], flags, j[2]), jobs_list))
    correctness = [_obj_name(r) for r in CORRECTNESS_SOURCES + CORRECTNESS_CUDA_SOURCES]
    _link(outs["correctness_framework_tests"],
          [_obj_name("tests/correctness_framework_tests.cpp")] + correctness)
    _link(outs["operator_api_tests"], [_obj_name("operator_api_tests_sm100.cpp")] + correctness)
    _link(outs["chain_harness"],
          [_obj_name("harness_chain_harness.cpp"), _obj_name("harness_research_stubs.cpp")] +
          [_obj_name(r) for r in BENCHMARK_SOURCES] + correctness)
    # Only the programs stay: no object or adapted reference source is kept.
    shutil.rmtree(os.path.join(OUT, "obj"))
    shutil.rmtree(os.path.join(OUT, "src"))
    return outs


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=None)
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build_harness(a.reference, a.force))
    return 0


if __name__ == "__main__":
    sys.exit(main())
