"""Generates the committed golden fixtures from RaggedRoute's own CPU reference
functions (oracle/_ref/librr_ref.so, compiled from the reference sources by
oracle/build_oracle.py). Run in the build container, where the reference
checkout exists:  python tests/golden/make_golden.py

Fixtures (small, seeded):
* topk_c2_slice.npz   -- 512 rows of the C2 logits (exact ties every 32nd row,
                         a NaN in row 0) -> ids/weights of the reference's float
                         top-2 (include/raggedroute/benchmark/adapter_utils.h:363-418).
* chain_c1_small.npz  -- a reduced C1-style chain_from_tokens (T=64, K=64,
                         E=8, N=16): reference top-2 ids, histogram, scan and
                         the reference's double-precision chain output.
* permute_small.npz   -- ids/offsets with their stable route_pos, checked by
                         the reference's validate_permute.
"""
from __future__ import annotations

import ctypes
import math
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle.build_oracle import build_oracle, build_reference  # noqa: E402

build_oracle()
assert build_reference() is not None, "the reference checkout is required"
import oracle  # noqa: E402
from raggedroute_b200.workloads import c2_logits  # noqa: E402

F = ctypes.POINTER(ctypes.c_float)
D = ctypes.POINTER(ctypes.c_double)
I = ctypes.POINTER(ctypes.c_int32)
ref = oracle.ref


def ref_top2_f32(logits):
    t, e = logits.shape
    ids = np.empty((t, 2), np.int32)
    w = np.empty((t, 2), np.float32)
    assert ref.rr_ref_top2_f32(logits.ctypes.data_as(F), t, e, ids.ctypes.data_as(I),
                               w.ctypes.data_as(F)) == 0
    return ids, w


def ref_hist_scan(ids, e):
    c = np.empty(e, np.int32)
    assert ref.rr_ref_histogram(ids.ctypes.data_as(I), ids.size, e, c.ctypes.data_as(I)) == 0
    o = np.empty(e + 1, np.int32)
    assert ref.rr_ref_exclusive_scan(c.ctypes.data_as(I), e, o.ctypes.data_as(I)) == 0
    return c, o


def main():
    logits = np.ascontiguousarray(c2_logits()[:512])
    ids, w = ref_top2_f32(logits)
    np.savez_compressed(os.path.join(HERE, "topk_c2_slice.npz"), logits=logits, ids=ids,
                        weights=w)

    rng = np.random.default_rng(0)
    t, k, e, n = 64, 64, 8, 16
    x = rng.uniform(-1, 1, (t, k)).astype(np.float32)
    wr = rng.normal(0, 1 / math.sqrt(k), (k, e)).astype(np.float32)
    we = rng.normal(0, 1 / math.sqrt(k), (e, k, n)).astype(np.float32)
    lg = oracle.chain_logits_f32(x, wr)
    cids, cw = ref_top2_f32(lg)
    counts, offsets = ref_hist_scan(np.ascontiguousarray(cids.reshape(-1)), e)
    y = np.empty((t, n), np.float32)
    assert ref.rr_ref_chain_from_tokens(x.ctypes.data_as(F), wr.ctypes.data_as(F), None,
                                        we.ctypes.data_as(F), t, k, e, n, 1,
                                        y.ctypes.data_as(F)) == 0
    np.savez_compressed(os.path.join(HERE, "chain_c1_small.npz"), x=x, router_w=wr, expert_w=we,
                        ids=cids, weights=cw, counts=counts, offsets=offsets, y_ref_f64=y)

    tokens, experts, top_k, hidden = 300, 16, 2, 8
    px = rng.uniform(-1, 1, (tokens, hidden)).astype(np.float32)
    pids = rng.integers(0, experts, tokens * top_k).astype(np.int32)
    _, poff = ref_hist_scan(pids, experts)
    xp, pos, sr, cur = oracle.stable_permute(px, pids, poff, experts, top_k)
    assert ref.rr_ref_validate_permute(px.ctypes.data_as(F), pids.ctypes.data_as(I),
                                       poff.ctypes.data_as(I), experts, xp.ctypes.data_as(F),
                                       pos.ctypes.data_as(I), sr.ctypes.data_as(I), tokens,
                                       top_k, hidden) == 1
    np.savez_compressed(os.path.join(HERE, "permute_small.npz"), x=px, ids=pids, offsets=poff,
                        route_pos=pos, sorted_route=sr, cursors=cur)
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
