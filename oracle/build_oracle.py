"""Build recipe for the CPU oracle (TEST INFRASTRUCTURE ONLY).

* ``oracle/librr_oracle.so`` -- this repository's plain-C restatement
  (``oracle/rr_oracle.c``), built with gcc.
* ``oracle/_ref/librr_ref.so`` -- RaggedRoute's own CPU reference functions,
  compiled from the sources where they lie in the reference checkout, plus the
  ctypes shim ``oracle/ref_shim.cpp``. Built only when the reference checkout
  is present (the build container); GPU boxes use the prebuilt file, which
  travels with the working tree. Nothing is copied out of the reference.

Where the reference checkout lies: ``--reference PATH``, else the
``RAGGEDROUTE_REFERENCE`` environment variable, else a checkout named
``reference`` beside this repository's directory. If none of these holds the
reference sources, only the restatement is built.

Run: ``python oracle/build_oracle.py [--reference PATH]``.
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)


def reference_checkout() -> str:
    """The reference checkout: $RAGGEDROUTE_REFERENCE, else ``reference``
    beside the repository directory (it may not exist)."""
    env = os.environ.get("RAGGEDROUTE_REFERENCE")
    if env:
        return env
    return os.path.join(os.path.dirname(REPO), "reference")

# Reference translation units that hold the CPU oracle and its helpers.
REFERENCE_SOURCES = [
    "src/dense_gemm/cpu_reference/reference.cpp",
    "src/grouped_gemm/cpu_reference/reference.cpp",
    "src/histogram/cpu_reference/reference.cpp",
    "src/permute/cpu_reference/reference.cpp",
    "src/scan/cpu_reference/reference.cpp",
    "src/topk_gate/cpu_reference/reference.cpp",
    "src/unpermute/cpu_reference/reference.cpp",
    "src/correctness/reference_validation.cpp",
    "src/correctness/report.cpp",
]
# framework.cu holds checked_mul/checked_int32 etc. next to a dtype kernel, so
# it goes through nvcc.
REFERENCE_CUDA_SOURCES = ["src/correctness/framework.cu"]


def _run(cmd: list[str]) -> None:
    subprocess.run(cmd, check=True)


def _stale(target: str, sources: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources if os.path.exists(s))


def build_oracle(force: bool = False) -> str:
    src = os.path.join(HERE, "rr_oracle.c")
    out = os.path.join(HERE, "librr_oracle.so")
    if force or _stale(out, [src]):
        _run(["gcc", "-O2", "-std=c11", "-ffp-contract=off", "-fno-fast-math", "-fPIC",
              "-shared", src, "-o", out, "-lm"])
    return out


def build_reference(reference: str | None = None, force: bool = False) -> str | None:
    """Compile the reference's CPU oracle into oracle/_ref (None if absent)."""
    reference = reference or reference_checkout()
    out_dir = os.path.join(HERE, "_ref")
    out = os.path.join(out_dir, "librr_ref.so")
    if not os.path.isdir(os.path.join(reference, "src")):
        return out if os.path.exists(out) else None
    shim = os.path.join(HERE, "ref_shim.cpp")
    sources = [os.path.join(reference, s) for s in REFERENCE_SOURCES]
    cuda_sources = [os.path.join(reference, s) for s in REFERENCE_CUDA_SOURCES]
    if not force and not _stale(out, sources + cuda_sources + [shim]):
        return out
    os.makedirs(out_dir, exist_ok=True)
    inc = os.path.join(reference, "include")
    objs = []
    for s in sources + [shim]:
        rel = os.path.relpath(s, reference) if s.startswith(reference) else os.path.basename(s)
        o = os.path.join(out_dir, rel.replace(os.sep, "_") + ".o")
        _run(["g++", "-std=c++17", "-O2", "-fPIC", "-ffp-contract=off", "-I" + inc,
              "-I/usr/local/cuda/include", "-c", s, "-o", o])
        objs.append(o)
    for s in cuda_sources:
        o = os.path.join(out_dir, os.path.basename(s) + ".o")
        _run(["nvcc", "-std=c++17", "-O2", "-Xcompiler", "-fPIC", "-I" + inc,
              "-gencode", "arch=compute_100a,code=sm_100a", "-c", s, "-o", o])
        objs.append(o)
    _run(["g++", "-shared", "-o", out] + objs +
         ["-L/usr/local/cuda/lib64", "-lcudart", "-lpthread"])
    for o in objs:
        os.remove(o)
    return out


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=None,
                    help="reference checkout (default: $RAGGEDROUTE_REFERENCE, else ../reference)")
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args()
    print(build_oracle(args.force))
    print(build_reference(args.reference, args.force))
    return 0


if __name__ == "__main__":
    sys.exit(main())
