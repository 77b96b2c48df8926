"""Route traces ("raggedroute.route_trace.v1") for chain_from_logits and
chain_from_route_ids: real routing working sets instead of synthetic ids.

The text form (.rrtrace) is read by the library (rr_route_trace_read, the
reference loader's validation: include/raggedroute/benchmark/adapter_utils.h:
250-322); the JSON form of the same schema
(configs/workloads/route_trace.schema.json) is read here with the same
checks. `trace_logits` builds the logits that make the top-2 gate select a
frame's ids (benchmarks/adapters/chain_adapter.cpp:222-228).
"""
from __future__ import annotations

import ctypes
import dataclasses
import json
import re

import numpy as np

from raggedroute_b200._lib import RRRouteTraceInfo, check, lib

SCHEMA = "raggedroute.route_trace.v1"
SOURCE_KINDS = ("production", "captured", "synthetic_fixture")
_PORTABLE = re.compile(r"^[A-Za-z0-9._-]+$")


@dataclasses.dataclass
class RouteTraceFrame:
    trace_id: str
    source_kind: str
    frame_id: str
    tokens: int
    experts: int
    top_k: int
    frame_count: int
    expert_ids: np.ndarray  # [tokens, top_k] int32


def load_route_trace_frame(path: str, frame: int = 0) -> RouteTraceFrame:
    """One frame of a .rrtrace text file, validated by the library."""
    info = RRRouteTraceInfo()
    check(lib().rr_route_trace_read(str(path).encode(), frame, ctypes.byref(info), None, 0),
          "rr_route_trace_read")
    ids = np.empty((info.tokens, info.top_k), np.int32)
    check(lib().rr_route_trace_read(str(path).encode(), frame, ctypes.byref(info),
                                    ids.ctypes.data_as(ctypes.c_void_p), ids.size),
          "rr_route_trace_read")
    return RouteTraceFrame(info.trace_id.decode(), info.source_kind.decode(),
                           info.frame_id.decode(), info.tokens, info.experts, info.top_k,
                           info.frame_count, ids)


def load_route_trace_json(path: str, frame: int = 0,
                          max_experts: int = 1024) -> RouteTraceFrame:
    """One frame of the JSON form, with the text loader's checks."""
    with open(path) as f:
        doc = json.load(f)
    if doc.get("schema_version") != SCHEMA:
        raise ValueError("invalid route trace header")
    tid, kind = doc.get("trace_id", ""), doc.get("source_kind", "")
    t, e, k, frames = doc.get("tokens"), doc.get("experts"), doc.get("top_k"), doc.get("frames")
    if (not isinstance(tid, str) or not _PORTABLE.match(tid) or kind not in SOURCE_KINDS or
            not all(isinstance(v, int) for v in (t, e, k)) or t < 1 or e < 1 or
            e > max_experts or k < 1 or k > e or not isinstance(frames, list) or not frames or
            not 0 <= frame < len(frames)):
        raise ValueError("invalid route trace metadata")
    seen = set()
    chosen = None
    for i, fr in enumerate(frames):
        fid = fr.get("frame_id")
        if not isinstance(fid, str) or not _PORTABLE.match(fid) or fid in seen:
            raise ValueError("route trace frame id is invalid or duplicated")
        seen.add(fid)
        ids = np.asarray(fr.get("expert_ids", []), dtype=np.int64)
        if ids.size != t * k or ids.min() < 0 or ids.max() >= e:
            raise ValueError("route trace contains an invalid expert id")
        ids = ids.reshape(t, k)
        if any(len(set(row.tolist())) != k for row in ids):
            raise ValueError("route trace repeats an expert within one token")
        if i == frame:
            chosen = (fid, ids.astype(np.int32))
    return RouteTraceFrame(tid, kind, chosen[0], t, e, k, len(frames), chosen[1])


def write_route_trace(path: str, trace_id: str, source_kind: str, experts: int,
                      frames: dict[str, np.ndarray]) -> None:
    """Writes the text form (all frames share tokens and top_k)."""
    first = next(iter(frames.values()))
    t, k = first.shape
    with open(path, "w") as f:
        f.write(f"{SCHEMA}\n{trace_id}\n{source_kind}\n{t} {experts} {k} {len(frames)}\n")
        for fid, ids in frames.items():
            f.write(fid + " " + " ".join(str(int(v)) for v in np.asarray(ids).reshape(-1)) + "\n")


def trace_logits(expert_ids: np.ndarray, experts: int) -> np.ndarray:
    """Host logits [T, E] whose top-2 are the frame's two ids in order."""
    ids = np.ascontiguousarray(expert_ids, dtype=np.int32)
    if ids.ndim != 2 or ids.shape[1] != 2:
        raise ValueError("trace logits need a top-2 frame")
    out = np.empty((ids.shape[0], experts), np.float32)
    check(lib().rr_route_trace_logits(ids.ctypes.data_as(ctypes.c_void_p), ids.shape[0], experts,
                                      out.ctypes.data_as(ctypes.c_void_p)),
          "rr_route_trace_logits")
    return out
