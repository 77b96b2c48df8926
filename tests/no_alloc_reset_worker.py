"""Child process of tests/test_zz_no_alloc.py::test_no_alloc_after_device_reset.

Torch-free on purpose: device memory comes from the cuda-python runtime
bindings and the library is driven through its C ABI with ctypes, so that
resetting the device here leaves no other framework holding stale state.

Sequence: rr_token_permute and rr_token_permute_no_alloc on the same inputs
(twice), cudaDeviceReset, a check that the device's new primary context has a
new context id, rr_token_permute alone on fresh buffers (the library works
again after the reset), then both entry points again. Every call's outputs
must equal the numpy stable permute bit for bit. Prints OK and exits 0 on
success; any mismatch or error exits non-zero before further launches.
"""
from __future__ import annotations

import ctypes
import importlib.util
import os
import sys

import numpy as np
from cuda.bindings import driver as drv
from cuda.bindings import runtime as rt

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def _load_binding():
    path = os.path.join(ROOT, "raggedroute_b200", "_lib.py")
    spec = importlib.util.spec_from_file_location("rr_c_abi", path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules["rr_c_abi"] = mod
    spec.loader.exec_module(mod)
    return mod


ABI = _load_binding()
LIB = ABI.lib()
H2D = rt.cudaMemcpyKind.cudaMemcpyHostToDevice
D2H = rt.cudaMemcpyKind.cudaMemcpyDeviceToHost


def check(result, what: str):
    err = result[0] if isinstance(result, tuple) else result
    if err != rt.cudaError_t.cudaSuccess:
        raise SystemExit(f"{what}: {err}")
    return result[1] if isinstance(result, tuple) and len(result) > 1 else None


def context_id() -> int:
    err, ctx = drv.cuCtxGetCurrent()
    if err != drv.CUresult.CUDA_SUCCESS or int(ctx) == 0:
        raise SystemExit(f"no current context: {err}")
    err, cid = drv.cuCtxGetId(ctx)
    if err != drv.CUresult.CUDA_SUCCESS:
        raise SystemExit(f"cuCtxGetId: {err}")
    return int(cid)


class Buffers:
    def __init__(self):
        self.ptrs = []

    def alloc(self, nbytes: int) -> int:
        p = check(rt.cudaMalloc(max(nbytes, 4)), "cudaMalloc")
        self.ptrs.append(p)
        return int(p)

    def upload(self, a: np.ndarray) -> int:
        p = self.alloc(a.nbytes)
        check(rt.cudaMemcpy(p, a.ctypes.data, a.nbytes, H2D), "cudaMemcpy H2D")
        return p

    def free(self):
        for p in self.ptrs:
            check(rt.cudaFree(p), "cudaFree")
        self.ptrs = []


def download(p: int, shape, dtype) -> np.ndarray:
    out = np.empty(shape, dtype)
    check(rt.cudaMemcpy(out.ctypes.data, p, out.nbytes, D2H), "cudaMemcpy D2H")
    return out


def stable_permute(x, ids, experts, top_k):
    counts = np.bincount(ids, minlength=experts)
    offsets = np.concatenate([[0], np.cumsum(counts)]).astype(np.int32)
    order = np.argsort(ids, kind="stable")
    pos = np.empty(ids.size, np.int32)
    pos[order] = np.arange(ids.size, dtype=np.int32)
    xp = x[order // top_k]
    return offsets, pos, order.astype(np.int32), xp


def run(tokens: int, experts: int, hidden: int, seed: int, no_alloc: bool) -> None:
    top_k = 2
    rng = np.random.default_rng(seed)
    x = rng.uniform(-1, 1, (tokens, hidden)).astype(np.float32)
    ids = rng.integers(0, experts, tokens * top_k).astype(np.int32)
    offsets, pos_ref, sr_ref, xp_ref = stable_permute(x, ids, experts, top_k)
    b = Buffers()
    dx, dids, doff = b.upload(x), b.upload(ids), b.upload(offsets)
    routes = tokens * top_k
    entries = [("rr_token_permute", LIB.rr_token_permute)]
    if no_alloc:
        entries.append(("rr_token_permute_no_alloc", LIB.rr_token_permute_no_alloc))
    for name, fn in entries:
        dxp = b.alloc(routes * hidden * 4)
        dpos, dsr = b.alloc(routes * 4), b.alloc(routes * 4)
        ws_bytes = LIB.rr_token_permute_workspace_size(tokens, experts, top_k, hidden)
        ws = b.alloc(ws_bytes) if name == "rr_token_permute" else 0
        ctx = ABI.RRContext(None, ws or None, ws_bytes if ws else 0, 0, 0, 0)
        st = fn(dx, dids, doff, dxp, dpos, dsr, tokens, experts, top_k, hidden, ctypes.byref(ctx))
        if st.code != 0:
            raise SystemExit(f"{name}: status {st.code} {st.message}")
        check(rt.cudaDeviceSynchronize(), f"{name} synchronize")
        if not np.array_equal(download(dpos, routes, np.int32), pos_ref):
            raise SystemExit(f"{name}: route_pos differs")
        if not np.array_equal(download(dsr, routes, np.int32), sr_ref):
            raise SystemExit(f"{name}: sorted_route differs")
        xp = download(dxp, (routes, hidden), np.float32)
        if not np.array_equal(xp.view(np.int32), xp_ref.view(np.int32)):
            raise SystemExit(f"{name}: rows differ")
    b.free()


def main() -> int:
    check(rt.cudaSetDevice(0), "cudaSetDevice")
    check(rt.cudaFree(0), "context init")
    first = context_id()
    run(3000, 64, 96, 1, no_alloc=True)
    run(40, 8, 12, 2, no_alloc=True)
    check(rt.cudaDeviceReset(), "cudaDeviceReset")
    check(rt.cudaSetDevice(0), "cudaSetDevice")
    check(rt.cudaFree(0), "context init after reset")
    second = context_id()
    if second == first:
        raise SystemExit("the reset kept the context id; not calling the no-alloc entry again")
    run(2000, 32, 64, 3, no_alloc=False)
    run(2000, 32, 64, 3, no_alloc=True)
    run(40, 8, 12, 4, no_alloc=True)
    print(f"OK contexts {first} -> {second}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
