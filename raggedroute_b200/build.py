"""Build recipe for libraggedroute_b200.so (sm_100a only).

Every .cu/.cpp file under raggedroute_b200/csrc is compiled by nvcc for
``-gencode arch=compute_100a,code=sm_100a`` and linked into
``raggedroute_b200/libraggedroute_b200.so`` in the source tree, so the library
travels with the working tree to the GPU host. The CUDA runtime and NCCL
(expert-parallel runtime) are linked dynamically: the library shares the
calling application's CUDA runtime, so kernels it launches into the caller's
streams and captured graphs are the caller's runtime objects (a caller can
inspect or update their graph nodes).

Usage: ``python -m raggedroute_b200.build [--force] [-j N]``.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(ROOT, "_build")
LIB = os.path.join(PKG, "libraggedroute_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC",
          "-I" + os.path.join(ROOT, "include"), "-I" + CSRC]
EXPORTS = os.path.join(CSRC, "exports.map")


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))


def headers() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) +
                  glob.glob(os.path.join(ROOT, "include", "*.h")) +
                  glob.glob(os.path.join(ROOT, "include", "raggedroute", "*.h")))


def _obj(src: str) -> str:
    return os.path.join(BUILD, os.path.basename(src) + ".o")


def _compile(src: str, verbose_ptxas: bool) -> str:
    out = _obj(src)
    cmd = [NVCC] + ARCH + COMMON + ["-c", src, "-o", out]
    if src.endswith(".cpp"):
        cmd[1:1] = ["-x", "cu"]
    if verbose_ptxas and src.endswith(".cu"):
        cmd += ["-Xptxas", "-v"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{res.stdout}\n{res.stderr}")
    if verbose_ptxas and res.stderr:
        sys.stderr.write(res.stderr)
    return out


def build(force: bool = False, jobs: int = 8, verbose_ptxas: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sources()
    newest_header = max((os.path.getmtime(h) for h in headers()), default=0.0)
    todo = []
    for s in srcs:
        o = _obj(s)
        if force or not os.path.exists(o) or os.path.getmtime(o) < max(os.path.getmtime(s),
                                                                        newest_header):
            todo.append(s)
    with cf.ThreadPoolExecutor(max_workers=max(1, jobs)) as ex:
        list(ex.map(lambda s: _compile(s, verbose_ptxas), todo))
    objs = [_obj(s) for s in srcs]
    if force or todo or not os.path.exists(LIB) or \
            os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        cmd = [NVCC] + ARCH + ["-shared", "-cudart", "shared", "-o", LIB] + objs + \
            ["-lnccl", "-lpthread", "-Xlinker", "--version-script=" + EXPORTS]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    return LIB


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=8)
    ap.add_argument("--ptxas-v", action="store_true", help="print register/smem usage")
    a = ap.parse_args()
    print(build(a.force, a.j, a.ptxas_v))
    return 0


if __name__ == "__main__":
    sys.exit(main())
