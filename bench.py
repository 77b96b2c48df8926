#!/usr/bin/env python
"""Benchmark: chain_from_tokens tokens/s on B200 (BASELINE.json `metric`).

Workload (N=1): BASELINE config C5 -- chain_from_tokens, FP32, T=65536
tokens per GPU, K=4096, E=128 experts, top-2, N=1408, router logits biased by
a log-Zipf(1.0) per-expert term; seeded synthetic inputs (no dataset exists
for this path). Every input is larger than the 126 MB L2 (X is 1 GiB, the
expert weights 2.95 GB), so no L2 flush is needed between steps.

One step = the seven-stage chain over one batch: dense_gemm -> topk_gate ->
histogram_exclusive_scan -> token_permute -> grouped_gemm -> unpermute, all
through libraggedroute_b200's C ABI on one stream. `value` is device-timed
(CUDA events, inputs resident in HBM, max over ranks); `e2e` is the same
metric with X in pinned host memory and Y returned to host memory every step
(one GPU: rr_chain_from_tokens_host, which overlaps the PCIe copies of
token chunks with the chain; expert parallelism: ep.HostPipeline, copy in,
EP step, copy out, with each step's copies overlapping its neighbours).
Extra keys on one GPU: `cold_scrub` (the C5 step with 256 MiB written to
flush L2 before every step), `small_configs` (C1 chain_from_tokens and C2
chain_from_logits latency, eager and replayed from a captured CUDA graph),
`configs` (C3 routing stages and C4 grouped GEMM, graph-timed) and
`prepared_weights` (the chain on expert weights prepared once, an inference
option).

Multi-GPU (torchrun): expert parallelism -- every rank runs its own T=65536
tokens (weak scaling); hot experts are replicated into virtual experts placed
by LPT on the measured loads, and rows move through the peer-memory
transport of rr_ep_chain_from_tokens (dispatch fused into the permute,
combine fused into the grouped GEMM epilogue; NCCL carries only the counts
and two one-word barriers per step).
--impl reference: times the reference's own CPU implementation of the path
(oracle/_ref, compiled from the reference sources) on bounded token samples of
the same workload, with every host thread; rank 0 only.
"""
from __future__ import annotations

import argparse
import ctypes
import dataclasses
import json

import numpy as np
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "chain_from_tokens tokens/s"
UNIT = "tokens/s"


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--tokens", type=int, default=None, help="override T per GPU (testing)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--gather-rows", action="store_true",
                    help="time the chain with the row-gathering grouped GEMM (no x_permuted); "
                         "implies --combine separate")
    ap.add_argument("--combine", choices=["fused", "separate"], default="fused",
                    help="fused: the unpermute runs in the grouped GEMM's epilogue "
                         "(rr_grouped_gemm_combine, y bit-identical); separate: grouped_gemm "
                         "then unpermute, as the reference's chain runs them")
    ap.add_argument("--no-extras", action="store_true",
                    help="skip the cold-L2 C5 pass and the C1/C2 eager-vs-graph latencies")
    ap.add_argument("--e2e-chunk", type=int, default=8192,
                    help="tokens per chunk of the host-memory chain (e2e, one GPU)")
    ap.add_argument("--ep-transport", choices=["auto", "peer", "nccl"], default="auto",
                    help="expert-parallel transport for --gpus > 1")
    ap.add_argument("--stages", action="store_true", help="print the per-stage table to stderr")
    ap.add_argument("--profile-once", action="store_true",
                    help="one warm-up chain, then one validated untimed chain_from_tokens call "
                         "(NVTX range per stage: raggedroute_<stage>) for profilers")
    ap.add_argument("--c3-permute", default=None, metavar="E:DIST[,E:DIST...]",
                    help="run only BASELINE C3's token_permute (R=1M routes, K=128) for the "
                         "given expert counts and id distributions, 3 calls each, and print "
                         "their event times: a small single-operator command for Nsight "
                         "Compute, e.g. 256:uniform,8:one")
    ap.add_argument("--gate-only", type=int, default=None, metavar="TOKENS",
                    help="run only topk_gate with bias at E=128 (C5's gate) over TOKENS rows "
                         "of N(0,1) logits, 3 calls each timed with CUDA events: a small "
                         "single-operator command for Nsight Compute (262144 rows = 134 MB "
                         "of logits, larger than L2)")
    ap.add_argument("--only-stage", default=None,
                    choices=["dense_gemm", "topk_gate", "histogram_exclusive_scan",
                             "token_permute", "grouped_gemm", "unpermute"],
                    help="profiling aid: run the chain once, then time only this stage")
    return ap.parse_args()


# ---------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------

class ClockSampler:
    """Samples nvidia-smi clocks/throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.proc = None
        self.lines: list[str] = []
        self._t = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.gpu_index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None
            return
        self._t = threading.Thread(target=self._read, daemon=True)
        self._t.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self._t is not None:
            self._t.join(timeout=2)
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() in ("active", "1"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------

def load_peaks() -> dict:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            p = json.load(f)
        p["source"] = "measured"
        return p
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def gemm_mixed_split(hidden: int) -> bool:
    """Whether the CTA-pair grouped GEMM runs the mixed split at this K (the
    library's rule: K >= 128 unless RAGGEDROUTE_B200_GEMM_MIXED=0)."""
    return hidden >= 128 and os.environ.get("RAGGEDROUTE_B200_GEMM_MIXED", "1")[:1] != "0"


def measure_tf32_peak(torch, device) -> float:
    """cuBLAS TF32 GEMM throughput (TFLOP/s) on this GPU, 8192^3, best of 10.
    The 3xTF32 roofline is this figure / 3."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    try:
        n = 8192
        a = torch.randn(n, n, device=device)
        b = torch.randn(n, n, device=device)
        for _ in range(3):
            torch.matmul(a, b)
        torch.cuda.synchronize()
        best = float("inf")
        for _ in range(10):
            s = torch.cuda.Event(enable_timing=True)
            e = torch.cuda.Event(enable_timing=True)
            s.record()
            torch.matmul(a, b)
            e.record()
            e.synchronize()
            best = min(best, s.elapsed_time(e))
        del a, b
        return 2.0 * n ** 3 / (best * 1e-3) / 1e12
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def load_traffic(name: str):
    """Per-launch DRAM traffic from the committed ncu summary, if present."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    if not os.path.exists(path):
        return None
    with open(path) as f:
        return json.load(f).get(name)


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------

def workload_config(tokens: int, world: int) -> dict:
    """The `config` object both arms report (BASELINE C5 per GPU)."""
    from raggedroute_b200.workloads import C5
    k, e, n = C5["hidden"], C5["experts"], C5["output"]
    return {"workload": f"C5 chain_from_tokens T={tokens}/GPU K={k} E={e} top2 N={n}",
            "tokens_per_gpu": tokens, "hidden": k, "experts": e, "output": n, "top_k": 2,
            "parallelism": f"ep{world}" if world > 1 else "single",
            "l2": "inputs larger than L2 (X 1 GiB, W 2.95 GB); no flush"}


def run_ours(args, rank: int, world: int, local_rank: int) -> dict | None:
    import torch
    import torch.distributed as dist

    import raggedroute_b200 as rr
    from raggedroute_b200.workloads import C5, c5_inputs

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    tokens = args.tokens or C5["tokens"]
    k, e, n = C5["hidden"], C5["experts"], C5["output"]
    routes = 2 * tokens
    inp = c5_inputs(device, tokens, rank=rank)
    buf = rr.ChainBuffers.allocate(tokens, k, e, n, device)
    stream = torch.cuda.Stream(device)
    ctx = rr.Context(stream=stream.cuda_stream)
    ep = None
    ep_info = None
    ep_buf = None
    if world > 1:
        # Expert parallelism with hot-expert replication: per-expert loads are
        # measured by routing this rank's batch (single-GPU stages), summed
        # over ranks, and turned into virtual experts placed by LPT.
        from raggedroute_b200.ep import ExpertParallel
        from raggedroute_b200.placement import ReplicatedPlacement
        rr.dense_gemm(inp.x, inp.router_w, buf.logits, tokens, e, k)
        rr.topk_gate_biased(buf.logits, inp.logit_bias, buf.expert_ids, buf.route_weights,
                            tokens, e)
        rr.histogram(buf.expert_ids, buf.counts, routes, e)
        loads = buf.counts.to(torch.float64)
        dist.all_reduce(loads)
        pl = ReplicatedPlacement(loads.cpu().numpy(), world)
        v_experts = pl.virtual_experts
        local = v_experts // world
        v2r = torch.from_numpy(pl.virtual_to_real[rank * local:(rank + 1) * local]).to(device)
        local_w = inp.expert_w[v2r].contiguous()
        remap = torch.from_numpy(pl.remap[rank]).to(device)
        ep = ExpertParallel(v_experts, tokens, k, n, timeout_s=300.0, router_experts=e,
                            transport=args.ep_transport)
        ep_buf = rr.ChainBuffers.allocate(tokens, k, v_experts, n, device, router_experts=e)
        ep_info = {"transport": ep.transport,
                   "placement": "replicated hot experts + LPT", "virtual_experts": v_experts,
                   "virtual_experts_per_rank": local,
                   "replicas_of_hottest": [int(r) for r in sorted(pl.replicas)[::-1][:4]],
                   "expected_imbalance": round(pl.imbalance(), 4)}
    torch.cuda.synchronize()

    fused = args.combine == "fused" and not args.gather_rows
    all_stages = ["dense_gemm", "topk_gate", "histogram_exclusive_scan", "token_permute",
                  "grouped_gemm", "unpermute"]
    # fused: the unpermute runs in the grouped GEMM's epilogue (y zeroed
    # first, each output row weighted and added into its token's row).
    stage_names = all_stages[:-1] if fused else all_stages
    # --gather-rows: the permute only ranks (route_pos, sorted_route) and the
    # grouped GEMM gathers its rows from X; x_permuted is never written.
    sorted_route = torch.empty(routes, dtype=torch.int32, device=device)

    def step(events=None, only=None, fused=fused):
        """One chain step, stage by stage; `only` runs just that stage index."""
        calls = [
            lambda: rr.dense_gemm(inp.x, inp.router_w, buf.logits, tokens, e, k, ctx=ctx),
            lambda: rr.topk_gate_biased(buf.logits, inp.logit_bias, buf.expert_ids,
                                        buf.route_weights, tokens, e, ctx=ctx),
            lambda: rr.histogram_exclusive_scan(buf.expert_ids, buf.counts, buf.offsets, routes,
                                                e, ctx=ctx),
            (lambda: rr.token_permute(inp.x, buf.expert_ids, buf.offsets, buf.x_permuted,
                                      buf.route_pos, sorted_route if fused else None, tokens, e,
                                      2, k, buf.workspace, ctx=ctx)) if not args.gather_rows else
            (lambda: rr.token_permute(None, buf.expert_ids, buf.offsets, None, buf.route_pos,
                                      sorted_route, tokens, e, 2, 0, buf.workspace, ctx=ctx)),
            (lambda: rr.grouped_gemm_combine(buf.x_permuted, inp.expert_w, buf.offsets,
                                             sorted_route, buf.route_weights, buf.y, routes, 2,
                                             ctx=ctx)) if fused else
            (lambda: rr.grouped_gemm(buf.x_permuted, inp.expert_w, buf.offsets, buf.y_permuted,
                                     e, k, n, routes, ctx=ctx)) if not args.gather_rows else
            (lambda: rr.grouped_gemm_gather(inp.x, sorted_route, 2, inp.expert_w, buf.offsets,
                                            buf.y_permuted, routes, ctx=ctx)),
            lambda: rr.unpermute(buf.y_permuted, buf.route_pos, buf.route_weights, buf.y, tokens,
                                 2, n, ctx=ctx),
        ][:len(all_stages) - (1 if fused else 0)]
        for i, call in enumerate(calls):
            if only is not None and i != only:
                continue
            if events is not None:
                events[i].record(stream)
            call()
            if events is not None:
                events[i + 1].record(stream)

    if args.only_stage is not None:
        return run_only_stage(args, torch, rr, stream, step, stage_names, tokens, e, k, n, buf)
    if args.profile_once:
        return run_profile_once(torch, rr, stream, ctx, inp, buf, tokens, e)

    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(7)] for _ in range(args.steps)]

    def ep_step():
        ep.chain_from_tokens(inp.x, inp.router_w, local_w, ep_buf, logit_bias=inp.logit_bias,
                             expert_remap=remap, ctx=ctx)

    if ep is not None:
        # Per-stage kernel times of this GPU's workload come from an untimed
        # stage-by-stage pass of the single-GPU chain (same kernels).
        with torch.cuda.stream(stream):
            for i in range(args.steps):
                step(ev[i])
        stream.synchronize()

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step() if ep is None else ep_step()
    stream.synchronize()

    launches0 = rr.kernel_launch_count()
    clocks = ClockSampler(local_rank)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    start = torch.cuda.Event(enable_timing=True)
    stop = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        start.record(stream)
        for i in range(args.steps):
            step(ev[i]) if ep is None else ep_step()
        stop.record(stream)
    stop.synchronize()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clock_info = clocks.stop()
    launches = rr.kernel_launch_count() - launches0
    total_ms = start.elapsed_time(stop)
    stage_ms = {nm: statistics.mean(ev[i][j].elapsed_time(ev[i][j + 1])
                                    for i in range(args.steps))
                for j, nm in enumerate(stage_names)}
    if ep is not None:
        sent, received = ep.last_step_rows()
        rows = torch.tensor([received], device=device, dtype=torch.float64)
        gathered = [torch.zeros_like(rows) for _ in range(world)]
        dist.all_gather(gathered, rows)
        per_rank = [int(g.item()) for g in gathered]
        ep_info["rows_received_per_rank"] = per_rank
        ep_info["measured_imbalance"] = round(max(per_rank) / (sum(per_rank) / world), 4)

    # The same step with the separate unpermute (the reference chain's
    # order of launches), timed the same way, and its y against the fused
    # step's bit for bit.
    separate = None
    if fused and world == 1 and not args.no_extras:
        y_fused = buf.y.clone()
        sev = [[torch.cuda.Event(enable_timing=True) for _ in range(7)]
               for _ in range(args.steps)]
        with torch.cuda.stream(stream):
            for _ in range(args.warmup):
                step(fused=False)
        stream.synchronize()
        a0 = torch.cuda.Event(enable_timing=True)
        a1 = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            a0.record(stream)
            for i in range(args.steps):
                step(sev[i], fused=False)
            a1.record(stream)
        a1.synchronize()
        sep_ms = a0.elapsed_time(a1) / args.steps
        separate = {
            "ms_per_step": round(sep_ms, 4),
            "tokens_per_s": round(tokens / (sep_ms * 1e-3), 1),
            "grouped_gemm_ms": round(statistics.mean(sev[i][4].elapsed_time(sev[i][5])
                                                     for i in range(args.steps)), 4),
            "unpermute_ms": round(statistics.mean(sev[i][5].elapsed_time(sev[i][6])
                                                  for i in range(args.steps)), 4),
            "y_bit_identical_to_fused": bool(torch.equal(y_fused.view(torch.int32),
                                                         buf.y.view(torch.int32))),
        }
        del y_fused

    # Max over ranks.
    t = torch.tensor([total_ms], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    max_ms = float(t.item())
    value = tokens * world * args.steps / (max_ms * 1e-3)

    # Correctness of the timed configuration (cheap exact checks).
    counts = buf.counts.cpu()
    assert int(counts.sum()) == routes

    # End-to-end through the public API with host buffers: one GPU uses the
    # host-memory chain (rr_chain_from_tokens_host: chunks of X in, the chain,
    # chunks of Y out, copies overlapped with the chain); expert parallelism
    # copies X in, runs the EP step and copies Y out.
    e2e = None
    if not args.no_e2e:
        x_host = inp.x.cpu().pin_memory()
        y_host = torch.empty(tokens, n, dtype=torch.float32).pin_memory()
        if ep is None:
            # x_host is written once before timing, so back-to-back steps may
            # overlap (the next step's copies in run while this one finishes).
            host_chain = rr.HostChain(args.e2e_chunk, k, e, n, input_ready=True)
        else:
            from raggedroute_b200.ep import HostPipeline
            ep_host = HostPipeline(ep, ep_buf, tokens, device)

        # The host chain runs the same kernels as the timed step (the fused
        # combine through the chain's implementation bits).
        host_ctx = dataclasses.replace(ctx, implementation_id=4 if fused else 0)

        def e2e_step():
            if ep is None:
                host_chain(x_host, inp.router_w, inp.expert_w, y_host,
                           logit_bias=inp.logit_bias, ctx=host_ctx)
                return
            ep_host(x_host, inp.router_w, local_w, y_host, logit_bias=inp.logit_bias,
                    expert_remap=remap, ctx=ctx)

        with torch.cuda.stream(stream):
            for _ in range(max(1, args.warmup)):
                e2e_step()
        stream.synchronize()
        if world > 1:
            dist.barrier()
        s2 = torch.cuda.Event(enable_timing=True)
        e2 = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            s2.record(stream)
            for _ in range(args.steps):
                e2e_step()
            e2.record(stream)
        e2.synchronize()
        te = torch.tensor([s2.elapsed_time(e2)], device=device, dtype=torch.float64)
        if world > 1:
            dist.all_reduce(te, op=dist.ReduceOp.MAX)
        # The PCIe bound of this number: one step's input copied from pinned
        # host memory to the device alone, best of 3 (CUDA events).
        x_dev = torch.empty_like(inp.x)
        h2d_ms = []
        with torch.cuda.stream(stream):
            for _ in range(3):
                c0 = torch.cuda.Event(enable_timing=True)
                c1 = torch.cuda.Event(enable_timing=True)
                c0.record(stream)
                x_dev.copy_(x_host, non_blocking=True)
                c1.record(stream)
                c1.synchronize()
                h2d_ms.append(c0.elapsed_time(c1))
        del x_dev
        h2d_gbs = x_host.numel() * 4 / (min(h2d_ms) * 1e-3) / 1e9
        e2e = {"value": tokens * world * args.steps / (float(te.item()) * 1e-3), "unit": UNIT,
               "h2d_bytes_per_step": x_host.numel() * 4,
               "d2h_bytes_per_step": y_host.numel() * 4,
               "h2d_gbs_measured": round(h2d_gbs, 2),
               "h2d_bound_tokens_per_s": round(tokens * world / (x_host.numel() * 4 / (h2d_gbs * 1e9)),
                                               1),
               "api": ("rr_chain_from_tokens_host (input-ready plan: consecutive steps "
                       "overlap), chunk %d tokens" % args.e2e_chunk
                       if ep is None else "raggedroute_b200.ep.HostPipeline: copy in, "
                       "rr_ep_chain_from_tokens, copy out, overlapped across steps")}
        if ep is None:
            host_chain.close()

    if ep is not None:
        ep.close()
    plain = None
    if ep is not None and not args.no_extras:
        plain = ep_plain_sharding(torch, dist, rr, args, inp, tokens, k, e, n, world, rank,
                                  device, stream, ctx)
    extras = {}
    if separate is not None:
        extras["separate_unpermute"] = separate
    if world == 1 and not args.no_extras:
        cold = cold_scrub_step(torch, rr, stream, step, max(3, args.steps))
        cold["tokens_per_s"] = round(tokens / (cold["ms_per_step"] * 1e-3), 1)
        extras["cold_scrub"] = cold
        extras["small_configs"] = small_config_latency(torch, rr, device)
    if rank != 0:
        return None

    peaks = load_peaks()
    tf32 = measure_tf32_peak(torch, device)
    # Ceilings from the measured dense bf16 peak, in bf16-MMA units per
    # product (TF32 runs at half the bf16 rate on this part): the mixed split
    # the grouped GEMM runs (hi.hi in TF32 = 2 units, two bfloat16 corrections
    # = 2 units) is bf16 / 4; the 3xTF32 split (3 TF32 products = 6 units),
    # kept for reference and for the one-CTA engine, is bf16 / 6.
    mixed = gemm_mixed_split(k)
    div = 4.0 if mixed else 6.0
    peak_3x = float(peaks["bf16_tflops"]) / 6.0
    peak_split = float(peaks["bf16_tflops"]) / div
    peak_split_sustained = float(peaks.get("bf16_tflops_sustained",
                                           peaks["bf16_tflops"])) / div
    gemm_flops = 2.0 * routes * k * n
    gemm_ms = stage_ms["grouped_gemm"]
    achieved = gemm_flops / (gemm_ms * 1e-3) / 1e12
    hbm = float(peaks["hbm_gbs"])
    stage_bytes = {
        "dense_gemm": 4.0 * (tokens * k + k * e + tokens * e),
        "topk_gate": 4.0 * tokens * e + 16.0 * tokens,
        "histogram_exclusive_scan": 4.0 * routes + 8.0 * e + 4,
        "token_permute": 4.0 * tokens * k + 4.0 * routes * k + 8.0 * routes + 4.0 * (e + 1),
        "grouped_gemm": 4.0 * (routes * k + e * k * n + routes * n),
        "unpermute": 4.0 * routes * n + 8.0 * routes + 4.0 * tokens * n,
    }
    if args.gather_rows:
        # ranks only: ids read, route_pos and sorted_route written
        stage_bytes["token_permute"] = 12.0 * routes + 4.0 * (e + 1)
    if fused:
        # permute also writes sorted_route; the GEMM writes y (not
        # y_permuted) and reads each row's route and weight.
        stage_bytes["token_permute"] += 4.0 * routes
        stage_bytes["grouped_gemm"] = 4.0 * (routes * k + e * k * n + tokens * n) + 8.0 * routes
    if world == 1 and not args.no_extras:
        extras["configs"] = config_sweep(torch, rr, device, hbm, peak_3x,
                                         float(peaks["bf16_tflops"]))
        extras["prepared_weights"] = prepared_weights_pass(
            torch, rr, stream, inp, buf, tokens, max(3, args.steps), gemm_flops, peak_3x)
    stages = {}
    for nm in stage_names:
        ms = stage_ms[nm]
        gbs = stage_bytes[nm] / (ms * 1e-3) / 1e9
        entry = {"ms": round(ms, 4), "GB/s": round(gbs, 1), "hbm_frac": round(gbs / hbm, 3)}
        if nm == "grouped_gemm":
            entry["TFLOP/s"] = round(achieved, 2)
            entry["tensor_frac"] = round(achieved / peak_split, 3)
            entry["split"] = "mixed (TF32 hi.hi + bf16 corrections)" if mixed else "3xTF32"
        if nm == "dense_gemm":
            df = 2.0 * tokens * k * e / (ms * 1e-3) / 1e12
            entry["TFLOP/s"] = round(df, 2)
        stages[nm] = entry
    if args.stages:
        print(json.dumps(stages, indent=1), file=sys.stderr)

    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": max_ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None,
        "dtype": ("f32 (GEMMs: TF32 hi.hi + bf16 correction products)"
                  if mixed else "f32 (3xTF32 GEMMs)"),
        "data": "synthetic (seeded; BASELINE C5 shapes and distributions)",
        "config": workload_config(tokens, world),
        "roofline": {"bound": "tensor", "kernel": "grouped_gemm", "achieved": round(achieved, 2),
                     "peak": round(peak_split, 2), "unit": "TFLOP/s",
                     "frac": round(achieved / peak_split, 4),
                     "peak_source": (
                         ("MEASURED_PEAKS bf16_tflops %.1f (%s) / 4 (mixed split: one TF32 "
                          "product at half the bf16 rate + two bf16 products)"
                          if mixed else
                          "MEASURED_PEAKS bf16_tflops %.1f (%s) / 2 (TF32 rate) / 3 "
                          "(MMAs per product)") % (float(peaks["bf16_tflops"]), peaks["source"])),
                     "frac_of_sustained": round(achieved / peak_split_sustained, 4),
                     "frac_of_3xtf32_ceiling": round(achieved / peak_3x, 4),
                     "cublas_tf32_live_tflops": round(tf32, 1),
                     "frac_of_cublas_tf32_ceiling": round(achieved / (tf32 / (div / 2.0)), 4),
                     "traffic": load_traffic("grouped_gemm")},
        "stages": stages,
        "clocks": clock_info,
        "gpu_launches": int(launches),
        "e2e": e2e,
    }
    line["path"] = ("operator calls through the C ABI on one stream: dense_gemm, "
                    "topk_gate_biased, histogram_exclusive_scan, token_permute, " +
                    ("grouped_gemm_combine (the unpermute fused into the grouped GEMM's epilogue; "
                     "y bit-identical to grouped_gemm + unpermute)" if fused else
                     "grouped_gemm, unpermute"))
    line.update(extras)
    if ep_info is not None:
        line["ep"] = ep_info
        line["config"]["placement"] = {
            "experts_per_gpu_plain": e // world,
            "virtual_experts": ep_info["virtual_experts"],
            "virtual_experts_per_gpu": ep_info["virtual_experts_per_rank"],
            "replicas_of_hottest": ep_info["replicas_of_hottest"],
            "rule": "hot experts replicated, copies placed by LPT (the timed value); BASELINE's "
                    "plain sharding is timed beside it under ep_plain_sharding",
            "transport": ep_info["transport"]}
        if plain is not None:
            line["ep_plain_sharding"] = plain
        line["roofline"]["note"] = ("per-GPU stage pass of the single-GPU chain on rank 0's "
                                    "tokens (same kernels), untimed region")
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(inp, steps=1)
    return line


def run_only_stage(args, torch, rr, stream, step, stage_names, tokens, e, k, n, buf) -> dict:
    """Runs the whole chain once (untimed setup), then `steps` launches of one
    stage through the same C ABI call the chain uses; reports its mean time.
    Meant as a small, single-kernel command for Nsight Compute."""
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(7)]
    with torch.cuda.stream(stream):
        step(ev)
    stream.synchronize()
    idx = stage_names.index(args.only_stage)
    times = []
    for _ in range(max(1, args.steps)):
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(7)]
        with torch.cuda.stream(stream):
            step(evs, only=idx)
        stream.synchronize()
        times.append(evs[idx].elapsed_time(evs[idx + 1]))
    counts = buf.counts.cpu()
    nonempty = int((counts > 0).sum())
    rows = int(counts.sum())
    # Algorithmic DRAM bytes of the fused grouped GEMM at this size: x_permuted
    # rows and the weights of the experts that have rows read once, y written
    # once, route and weight read per row (so a capture's traffic can be set
    # against its own size).
    gemm_bytes = 4.0 * (rows * k + nonempty * k * n + tokens * n) + 8.0 * rows
    return {"stage": args.only_stage, "tokens": tokens, "ms": statistics.mean(times),
            "ms_min": min(times), "rows": rows, "nonempty_experts": nonempty,
            "grouped_gemm_algorithmic_bytes": gemm_bytes}


def ep_plain_sharding(torch, dist, rr, args, inp, tokens, k, e, n, world, rank, device, stream,
                      ctx) -> dict:
    """BASELINE C5's plain expert sharding (experts [g*E/N, (g+1)*E/N) on GPU g,
    no replicas), timed like the main value: warm-up, barrier, K steps
    between CUDA events on the launching stream, max over ranks."""
    from raggedroute_b200.ep import ExpertParallel
    local = e // world
    w = inp.expert_w[rank * local:(rank + 1) * local].contiguous()
    plan = ExpertParallel(e, tokens, k, n, timeout_s=300.0, router_experts=e,
                          transport=args.ep_transport)
    b = rr.ChainBuffers.allocate(tokens, k, e, n, device, router_experts=e)

    def one_step():
        plan.chain_from_tokens(inp.x, inp.router_w, w, b, logit_bias=inp.logit_bias, ctx=ctx)

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            one_step()
    stream.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    a0 = torch.cuda.Event(enable_timing=True)
    a1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        a0.record(stream)
        for _ in range(args.steps):
            one_step()
        a1.record(stream)
    a1.synchronize()
    t = torch.tensor([a0.elapsed_time(a1)], device=device, dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms = float(t.item()) / args.steps
    _, received = plan.last_step_rows()
    rows = torch.tensor([received], device=device, dtype=torch.float64)
    gathered = [torch.zeros_like(rows) for _ in range(world)]
    dist.all_gather(gathered, rows)
    per_rank = [int(g.item()) for g in gathered]
    plan.close()
    del b, w
    return {"placement": f"experts [g*{local}, (g+1)*{local}) on GPU g, no replicas",
            "tokens_per_s": round(tokens * world / (ms * 1e-3), 1), "ms_per_step": round(ms, 4),
            "rows_received_per_rank": per_rank,
            "measured_imbalance": round(max(per_rank) / (sum(per_rank) / world), 4)}


def run_c3_permute(spec: str) -> dict:
    """C3's stable token_permute (R = 1,048,576 routes, T = R/2 tokens, K = 128,
    with sorted_route) for each E:dist in spec: histogram + scan once, then
    three permute calls, each timed with CUDA events; nothing else runs."""
    import torch

    import raggedroute_b200 as rr
    from raggedroute_b200.workloads import C3, route_ids
    device = torch.device("cuda", 0)
    routes, k = C3["routes"], C3["hidden"]
    tokens = routes // 2
    x = torch.rand(tokens, k, device=device) * 2 - 1
    xp = torch.empty(routes, k, device=device)
    pos = torch.empty(routes, dtype=torch.int32, device=device)
    srt = torch.empty(routes, dtype=torch.int32, device=device)
    out = {}
    for item in spec.split(","):
        e_s, dist = item.split(":")
        e = int(e_s)
        counts = torch.empty(e, dtype=torch.int32, device=device)
        offsets = torch.empty(e + 1, dtype=torch.int32, device=device)
        ws = torch.empty(rr.token_permute_workspace_size(tokens, e, 2, k) // 4 + 1,
                         dtype=torch.int32, device=device)
        ids = torch.as_tensor(route_ids(routes, e, dist, seed=C3["seed"]), device=device)
        rr.histogram_exclusive_scan(ids, counts, offsets, routes, e)
        times = []
        for _ in range(3):
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record()
            rr.token_permute(x, ids, offsets, xp, pos, srt, tokens, e, 2, k, ws)
            b.record()
            b.synchronize()
            times.append(a.elapsed_time(b) * 1e3)
        out[f"E{e}_{dist}"] = {"token_permute_us": [round(t, 2) for t in times]}
    return {"c3_permute": out}


def run_gate_only(tokens: int) -> dict:
    """C5's topk_gate (E = 128, per-expert bias) over `tokens` rows of N(0,1)
    logits: three calls, each timed with CUDA events; nothing else runs."""
    import torch

    import raggedroute_b200 as rr
    device = torch.device("cuda", 0)
    e = 128
    g = torch.Generator(device=device)
    g.manual_seed(4)
    logits = torch.randn(tokens, e, generator=g, device=device)
    bias = torch.randn(e, generator=g, device=device)
    ids = torch.empty(tokens, 2, dtype=torch.int32, device=device)
    w = torch.empty(tokens, 2, device=device)
    times = []
    for _ in range(3):
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record()
        rr.topk_gate_biased(logits, bias, ids, w, tokens, e)
        b.record()
        b.synchronize()
        times.append(a.elapsed_time(b) * 1e3)
    return {"gate_only": {"tokens": tokens, "experts": e,
                          "bytes": 4 * tokens * e + 16 * tokens,
                          "topk_gate_us": [round(t, 2) for t in times]}}


def run_profile_once(torch, rr, stream, ctx, inp, buf, tokens: int, e: int) -> dict:
    """One warm-up chain, then exactly one untimed chain_from_tokens call for a
    profiler (the library brackets each stage in an NVTX range named
    raggedroute_<stage>), validated by the routing invariants: ids in [0, E),
    counts summing to 2T, offsets their exclusive scan, y finite."""
    for _ in range(2):
        with torch.cuda.stream(stream):
            rr.chain_from_tokens(inp.x, inp.router_w, inp.expert_w, buf,
                                 logit_bias=inp.logit_bias, ctx=ctx)
        stream.synchronize()
    ids = buf.expert_ids
    counts = buf.counts.to(torch.int64)
    ok = (bool(((ids >= 0) & (ids < e)).all()) and int(counts.sum()) == 2 * tokens
          and int(buf.offsets[0]) == 0
          and torch.equal(buf.offsets[1:].to(torch.int64), torch.cumsum(counts, 0))
          and bool(torch.isfinite(buf.y).all()))
    if not ok:
        raise RuntimeError("profile-once chain failed its routing invariants")
    return {"profile_once": True, "tokens": tokens, "validated": ok}


def small_config_latency(torch, rr, device, iters: int = 200) -> dict:
    """C1 (chain_from_tokens) and C2 (chain_from_logits) per-call latency,
    launched eagerly and as a captured CUDA graph (rr_graph_*), CUDA events
    over `iters` back-to-back calls on one stream."""
    from raggedroute_b200.workloads import C1, C2, c1_inputs, c2_inputs
    out = {}
    for cfg, make, logits_mode in ((C1, c1_inputs, False), (C2, c2_inputs, True)):
        inp = make(device)
        t, k, e, n = cfg["tokens"], cfg["hidden"], cfg["experts"], cfg["output"]
        buf = rr.ChainBuffers.allocate(t, k, e, n, device)
        stream = torch.cuda.Stream(device)
        if logits_mode:
            call = lambda ctx: rr.chain_from_logits(inp.logits, inp.x, inp.expert_w, buf,  # noqa: E731
                                                    ctx=ctx)
        else:
            call = lambda ctx: rr.chain_from_tokens(inp.x, inp.router_w, inp.expert_w, buf,  # noqa: E731
                                                    logit_bias=inp.logit_bias, ctx=ctx)
        ctx = rr.Context(stream=stream.cuda_stream)
        for _ in range(20):
            call(ctx)
        graph = rr.Graph.capture(call, stream)
        res = {}
        for mode in ("eager", "graph"):
            for _ in range(20):
                call(ctx) if mode == "eager" else graph.launch(stream)
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record(stream)
            for _ in range(iters):
                call(ctx) if mode == "eager" else graph.launch(stream)
            b.record(stream)
            b.synchronize()
            res[mode + "_us"] = round(a.elapsed_time(b) * 1e3 / iters, 2)
        res["graph_tokens_per_s"] = round(t / (res["graph_us"] * 1e-6), 1)
        res["graph_nodes"] = graph.nodes
        graph.close()
        out[cfg["name"]] = res
    return out


def cold_scrub_step(torch, rr, stream, step, steps: int) -> dict:
    """The C5 chain with the L2 scrubbed (256 MiB written) before every step;
    only the chain is inside the timed events."""
    scrub = torch.empty(64 << 20, dtype=torch.int32, device=stream.device)
    ctx_s = rr.Context(stream=stream.cuda_stream)
    total = 0.0
    for _ in range(steps):
        rr.lib().rr_launch_cache_scrub(ctypes.c_void_p(scrub.data_ptr()), scrub.numel(),
                                       ctypes.c_void_p(ctx_s.stream))
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            a.record(stream)
            step()
            b.record(stream)
        b.synchronize()
        total += a.elapsed_time(b)
    return {"ms_per_step": round(total / steps, 3), "scrub_bytes": scrub.numel() * 4}


def prepared_weights_pass(torch, rr, stream, inp, buf, tokens: int, steps: int,
                          gemm_flops: float, peak_3x: float) -> dict:
    """chain_from_tokens on expert weights prepared once (PreparedExpertWeights:
    K-major hi/lo, so the grouped GEMM loads all of B ready for its MMAs and
    splits only the token rows) -- an inference option next to the drop-in
    call, which the headline value measures. Reports the one-time
    preparation, the chain per step and the grouped GEMM alone, CUDA events on
    the same C5 inputs. An error here is reported, not raised."""
    try:
        ctx = rr.Context(stream=stream.cuda_stream)
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            a.record(stream)
            prep = rr.PreparedExpertWeights(inp.expert_w, ctx=ctx)
            b.record(stream)
        b.synchronize()
        prepare_ms = a.elapsed_time(b)

        def step():
            rr.chain_from_tokens(inp.x, inp.router_w, prep, buf, logit_bias=inp.logit_bias,
                                 ctx=ctx)

        with torch.cuda.stream(stream):
            for _ in range(3):
                step()
            a.record(stream)
            for _ in range(steps):
                step()
            b.record(stream)
        b.synchronize()
        chain_ms = a.elapsed_time(b) / steps
        with torch.cuda.stream(stream):
            a.record(stream)
            for _ in range(5):
                rr.grouped_gemm_prepared(buf.x_permuted, prep, buf.offsets, buf.y_permuted,
                                         2 * tokens, ctx=ctx)
            b.record(stream)
        b.synchronize()
        gemm_ms = a.elapsed_time(b) / 5
        tflops = gemm_flops / (gemm_ms * 1e-3) / 1e12
        del prep
        return {"prepare_ms": round(prepare_ms, 3), "ms_per_step": round(chain_ms, 3),
                "tokens_per_s": round(tokens / (chain_ms * 1e-3), 1),
                "grouped_gemm_ms": round(gemm_ms, 3), "grouped_gemm_TFLOP/s": round(tflops, 2),
                "tensor_frac_3xtf32": round(tflops / peak_3x, 3),
                "note": "expert weights prepared once (rr_prepare_expert_weights), an "
                        "inference option; `value` is the drop-in call on raw weights"}
    except Exception as ex:  # noqa: BLE001 - an optional extra must not cost the bench line
        return {"error": f"{type(ex).__name__}: {ex}"[:300]}


def _event_us(torch, rr, stream, fn, iters: int) -> float:
    """Mean device time of one fn(ctx) call in microseconds: `iters` calls are
    captured into one CUDA graph (rr_graph_*), so host call overhead does not
    starve the GPU between short kernels, and the replay is timed with CUDA
    events after 3 untimed calls and one untimed replay."""
    ctx = rr.Context(stream=stream.cuda_stream)
    with torch.cuda.stream(stream):
        for _ in range(3):
            fn(ctx)
    graph = rr.Graph.capture(lambda c: [fn(c) for _ in range(iters)], stream)
    try:
        graph.launch(stream)
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        graph.launch(stream)
        b.record(stream)
        b.synchronize()
    finally:
        graph.close()
    return a.elapsed_time(b) * 1e3 / iters


def config_sweep(torch, rr, device, hbm_gbs: float, peak_3x: float, bf16_tflops: float) -> dict:
    """The BASELINE parity configs C3 and C4 timed on their own (warm L2 as in
    the reference's protocol; device time per call from a captured graph of
    back-to-back calls, see _event_us).

    C3: 1,048,576 routes (T=524,288, K=128) for E in {1, 8, 64, 256} x ids
    {uniform, Zipf(1.5), all-to-one}: histogram, exclusive_scan, the fused
    histogram_exclusive_scan and the stable token_permute (with sorted_route;
    top_k = 2, so not at E = 1).
    Bytes per call are the algorithmic ones (ids read once; for the permute
    X read once, Xp written, ids, route_pos and sorted_route).
    C4: grouped_gemm over R=32768 rows, E=64 (6 empty, Zipf(1.1) sizes),
    K=N=1024; 2*R*K*N FLOP against the 3xTF32 peak."""
    from raggedroute_b200.workloads import C3, C4, c4_group_sizes, offsets_from_sizes, route_ids
    stream = torch.cuda.Stream(device)
    out = {}
    # The gate alone at C5 shapes (logits [65536, 128] + bias -> ids, weights).
    gt, ge = 65536, 128
    logits = torch.randn(gt, ge, device=device)
    bias = torch.randn(ge, device=device)
    g_ids = torch.empty(gt, 2, dtype=torch.int32, device=device)
    g_w = torch.empty(gt, 2, device=device)
    gate = _event_us(torch, rr, stream, lambda c: rr.topk_gate_biased(
        logits, bias, g_ids, g_w, gt, ge, ctx=c), 50)
    gate_b = 4.0 * gt * ge + 16.0 * gt
    # The floor of one launch in a graph: a one-expert scan (one tiny kernel).
    one_c = torch.ones(1, dtype=torch.int32, device=device)
    one_o = torch.empty(2, dtype=torch.int32, device=device)
    floor_us = _event_us(torch, rr, stream, lambda c: rr.exclusive_scan(one_c, one_o, 1, ctx=c), 50)
    out["C5_topk_gate"] = {"us": round(gate, 2),
                           "hbm_frac": round(gate_b / (gate * 1e-6) / 1e9 / hbm_gbs, 3),
                           "hbm_frac_above_launch_floor": round(
                               gate_b / (max(gate - floor_us, 1e-3) * 1e-6) / 1e9 / hbm_gbs, 3)}
    g_counts = torch.empty(ge, dtype=torch.int32, device=device)
    g_offsets = torch.empty(ge + 1, dtype=torch.int32, device=device)
    hs = _event_us(torch, rr, stream, lambda c: rr.histogram_exclusive_scan(
        g_ids, g_counts, g_offsets, 2 * gt, ge, ctx=c), 50)
    out["C5_histogram_exclusive_scan"] = {"us": round(hs, 2)}
    del logits
    routes, k = C3["routes"], C3["hidden"]
    tokens = routes // 2
    x = torch.rand(tokens, k, device=device) * 2 - 1
    xp = torch.empty(routes, k, device=device)
    pos = torch.empty(routes, dtype=torch.int32, device=device)
    srt = torch.empty(routes, dtype=torch.int32, device=device)
    c3 = {}
    out["launch_floor_us"] = round(floor_us, 2)
    for e in C3["experts"]:
        counts = torch.empty(e, dtype=torch.int32, device=device)
        offsets = torch.empty(e + 1, dtype=torch.int32, device=device)
        ws = torch.empty(rr.token_permute_workspace_size(tokens, e, 2, k) // 4 + 1,
                         dtype=torch.int32, device=device)
        for dist in ("uniform", "zipf", "one"):
            ids = torch.as_tensor(route_ids(routes, e, dist, seed=C3["seed"]), device=device)
            hist = _event_us(torch, rr, stream,
                             lambda c: rr.histogram(ids, counts, routes, e, ctx=c), 50)
            scan = _event_us(torch, rr, stream,
                             lambda c: rr.exclusive_scan(counts, offsets, e, ctx=c), 50)
            fused = _event_us(torch, rr, stream, lambda c: rr.histogram_exclusive_scan(
                ids, counts, offsets, routes, e, ctx=c), 50)
            # The two operators back to back in the same graph: the like-for-
            # like comparison for the fused one (separate graphs each carry
            # their own per-launch gaps).
            pair = _event_us(torch, rr, stream, lambda c: (
                rr.histogram(ids, counts, routes, e, ctx=c),
                rr.exclusive_scan(counts, offsets, e, ctx=c)), 50)
            hist_b = 4.0 * routes + 4.0 * e
            fused_b = 4.0 * routes + 8.0 * e + 4
            perm_b = 4.0 * tokens * k + 4.0 * routes * k + 12.0 * routes + 4.0 * (e + 1)

            def frac(b, us):
                return round(b / (us * 1e-6) / 1e9 / hbm_gbs, 3)

            # Above 256K routes the histogram is a memset and one kernel, the
            # fused operator a memset and two kernels.
            entry = {
                "histogram_us": round(hist, 2), "histogram_hbm_frac": frac(hist_b, hist),
                "histogram_hbm_frac_above_launch_floor":
                    frac(hist_b, max(hist - 2 * floor_us, 1e-3)),
                "exclusive_scan_us": round(scan, 2),
                "histogram_exclusive_scan_us": round(fused, 2),
                "histogram_then_exclusive_scan_us": round(pair, 2),
                "histogram_exclusive_scan_hbm_frac": frac(fused_b, fused)}
            if e >= 2:  # top_k = 2 needs two experts (the operator's top_k <= E rule)
                perm = _event_us(torch, rr, stream, lambda c: rr.token_permute(
                    x, ids, offsets, xp, pos, srt, tokens, e, 2, k, ws, ctx=c), 20)
                entry["token_permute_us"] = round(perm, 2)
                entry["token_permute_hbm_frac"] = frac(perm_b, perm)
            c3[f"E{e}_{dist}"] = entry
    out["C3"] = c3
    del x, xp, pos, srt
    r, e, k, n = C4["routes"], C4["experts"], C4["hidden"], C4["output"]
    sizes = c4_group_sizes(r, e, C4["empty"], seed=C4["seed"])
    offsets = torch.as_tensor(offsets_from_sizes(sizes), device=device)
    g = torch.Generator(device=device)
    g.manual_seed(C4["seed"])
    a = torch.rand(r, k, device=device, generator=g) * 2 - 1
    w = torch.randn(e, k, n, device=device, generator=g) / math.sqrt(k)
    y = torch.empty(r, n, device=device)
    gemm = _event_us(torch, rr, stream,
                     lambda c: rr.grouped_gemm(a, w, offsets, y, e, k, n, r, ctx=c), 20)
    tflops = 2.0 * r * k * n / (gemm * 1e-6) / 1e12
    c4_mixed = gemm_mixed_split(k)
    out["C4"] = {"grouped_gemm_us": round(gemm, 2), "TFLOP/s": round(tflops, 2),
                 "tensor_frac": round(tflops / (bf16_tflops / (4.0 if c4_mixed else 6.0)), 3),
                 "split": "mixed" if c4_mixed else "3xTF32",
                 "note": "W (256 MiB) and Xp (128 MiB) partly L2-resident between calls"}
    return out


# ---------------------------------------------------------------------------
# reference CPU arm
# ---------------------------------------------------------------------------

def _ref_lib():
    import oracle
    if oracle.ref is None:
        raise RuntimeError("oracle/_ref/librr_ref.so is missing (build it with "
                           "python oracle/build_oracle.py where the reference checkout exists)")
    return oracle.ref


def _sample_inputs(sample_tokens: int, device="cpu"):
    """Host copies of a C5 token sample plus the full router/expert weights."""
    import torch
    from raggedroute_b200.workloads import C5, c5_inputs
    gen_dev = "cuda" if torch.cuda.is_available() else "cpu"
    inp = c5_inputs(gen_dev, C5["tokens"])
    return (inp.x[:sample_tokens].contiguous().cpu(), inp.router_w.cpu(), inp.logit_bias.cpu(),
            inp.expert_w.cpu())


def _run_ref_chain(ref, x, wr, bias, we, threads):
    import ctypes
    import torch
    t, k = x.shape
    e = wr.shape[1]
    n = we.shape[2]
    y = torch.empty(t, n, dtype=torch.float32)
    f = ctypes.POINTER(ctypes.c_float)
    p = lambda a: ctypes.cast(a.data_ptr(), f)  # noqa: E731
    rc = ref.rr_ref_chain_from_tokens(p(x), p(wr), p(bias), p(we), t, k, e, n, threads, p(y))
    if rc != 0:
        raise RuntimeError("reference CPU chain failed")
    return y


def cpu_baseline(inp, steps: int = 1, sample_tokens: int = 256) -> dict:
    """The reference CPU chain on a bounded token sample (rank 0, N=1), timed
    at the sample size and at half of it: every stage's work is linear in the
    tokens (the GEMMs are per-token products, the routing stages per-route
    passes), so equal per-token times at both sizes support extrapolating to
    the full batch."""
    ref = _ref_lib()
    threads = os.cpu_count() or 1
    x = inp.x[:sample_tokens].contiguous().cpu()
    wr, bias, we = inp.router_w.cpu(), inp.logit_bias.cpu(), inp.expert_w.cpu()
    t0 = time.perf_counter()
    for _ in range(steps):
        _run_ref_chain(ref, x, wr, bias, we, threads)
    dt = (time.perf_counter() - t0) / steps
    half = max(1, sample_tokens // 2)
    th = time.perf_counter()
    _run_ref_chain(ref, x[:half].contiguous(), wr, bias, we, threads)
    dth = time.perf_counter() - th
    # The reference oracle as shipped is single-threaded: the same chain on
    # one host thread, on a smaller sample.
    one = max(1, sample_tokens // 16)
    t1 = time.perf_counter()
    _run_ref_chain(ref, x[:one].contiguous(), wr, bias, we, 1)
    dt1 = time.perf_counter() - t1
    return {"value": sample_tokens / dt, "unit": UNIT, "cores": threads, "kind": "reference",
            "sample": f"{sample_tokens} tokens of C5 per step through the reference's CPU "
                      f"functions (oracle/_ref), {threads} host threads, "
                      f"{dt:.1f} s of CPU work; the full batch is {C5_TOKENS} tokens",
            "linearity": {"tokens_per_s_at_sample": round(sample_tokens / dt, 2),
                          "tokens_per_s_at_half_sample": round(half / dth, 2),
                          "half_sample_tokens": half},
            "one_core": {"value": one / dt1, "unit": UNIT, "cores": 1,
                         "sample": f"{one} tokens of C5, 1 host thread"}}


C5_TOKENS = 65536


def run_reference(args, rank: int) -> dict | None:
    """Times the reference's CPU implementation of the path on bounded samples
    of the C5 workload: each step runs `sample` tokens through the reference
    CPU chain and the value is tokens per second (rank 0 only)."""
    if rank != 0:
        return None
    ref = _ref_lib()
    threads = os.cpu_count() or 1
    sample = int(os.environ.get("RR_REF_SAMPLE_TOKENS", "256"))
    x, wr, bias, we = _sample_inputs(sample)
    for _ in range(args.warmup):
        _run_ref_chain(ref, x, wr, bias, we, threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        _run_ref_chain(ref, x, wr, bias, we, threads)
    dt = (time.perf_counter() - t0) / args.steps
    value = sample / dt
    cpu = {"value": value, "unit": UNIT, "cores": threads, "kind": "reference",
           "sample": f"{sample} tokens of C5 per step through the reference's CPU functions "
                     f"(oracle/_ref), {threads} host threads"}
    return {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f64 (reference CPU oracle)", "data": "synthetic (seeded; C5 sample)",
            "config": workload_config(C5_TOKENS, args.gpus),
            "impl": "reference", "cpu_baseline": cpu,
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


def main() -> int:
    # Only the JSON line goes to stdout: libraries (NCCL prints its version on
    # communicator creation) write to stdout too, so fd 1 is pointed at stderr
    # for the run and the result is written to the saved descriptor.
    result_fd = os.dup(1)
    sys.stdout.flush()
    os.dup2(2, 1)
    try:
        line = _main()
    finally:
        sys.stdout.flush()
        os.dup2(result_fd, 1)
    if line is not None:
        os.write(result_fd, (json.dumps(line) + "\n").encode())
    os.close(result_fd)
    return 0


def _main() -> dict | None:
    args = parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank)
    if args.c3_permute is not None:
        return run_c3_permute(args.c3_permute)
    if args.gate_only is not None:
        return run_gate_only(args.gate_only)
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        return run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
