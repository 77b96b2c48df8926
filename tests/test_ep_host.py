"""Expert-parallel host logic on CPU (no GPU): placement, the per-rank
exchange plan (rr_ep_plan, C ABI), and a two-rank gloo run of the whole
protocol -- local routing, counts all-gather, plan, all-to-all dispatch,
per-(source, local expert) expert GEMMs, reverse all-to-all, unpermute --
with the oracle and numpy standing in for the device kernels. The two-rank
output must equal the single-process result for every token.
"""
from __future__ import annotations

import math
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_lpt_placement_balances_zipf():
    from raggedroute_b200.placement import (expected_loads_from_bias, imbalance, lpt_placement,
                                            relabel_permutation)
    from raggedroute_b200.workloads import zipf_log_bias
    e, g = 128, 8
    loads = expected_loads_from_bias(zipf_log_bias(e, 1.0))
    rank_of = lpt_placement(loads, g)
    assert np.all(np.bincount(rank_of, minlength=g) == e // g)
    contiguous = np.repeat(np.arange(g), e // g)
    assert imbalance(loads, rank_of, g) < imbalance(loads, contiguous, g)
    perm = relabel_permutation(rank_of)
    assert sorted(perm.tolist()) == list(range(e))
    # Relabelled experts of each rank are contiguous.
    assert np.all(rank_of[perm] == np.repeat(np.arange(g), e // g))


def test_ep_plan_matches_numpy(rrlib):
    from raggedroute_b200.ep import plan
    rng = np.random.default_rng(0)
    g, e = 4, 32
    counts = rng.integers(0, 50, (g, e)).astype(np.int32)
    local = e // g
    for rank in range(g):
        sr, so, rr_, ro = plan(counts, rank)
        exp_send = counts[rank].reshape(g, local).sum(axis=1)
        exp_recv = counts[:, rank * local:(rank + 1) * local].sum(axis=1)
        assert np.array_equal(sr, exp_send)
        assert np.array_equal(rr_, exp_recv)
        assert np.array_equal(so, np.concatenate([[0], np.cumsum(exp_send)[:-1]]))
        assert np.array_equal(ro, np.concatenate([[0], np.cumsum(exp_recv)[:-1]]))


def test_ep_plan_rejects_bad_shape(rrlib):
    from raggedroute_b200._lib import RaggedRouteError
    from raggedroute_b200.ep import plan
    with pytest.raises(RaggedRouteError):
        plan(np.zeros((3, 8), np.int32), 0)  # 8 experts over 3 ranks


T, K, E, N, G = 64, 16, 8, 12, 2


def _problem():
    rng = np.random.default_rng(123)
    xs = [rng.uniform(-1, 1, (T, K)).astype(np.float32) for _ in range(G)]
    wr = rng.normal(0, 1 / math.sqrt(K), (K, E)).astype(np.float32)
    we = rng.normal(0, 1 / math.sqrt(K), (E, K, N)).astype(np.float32)
    return xs, wr, we


def _ep_worker(rank: int, port: int, out_dir: str):
    import sys
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import torch
    import torch.distributed as dist

    import oracle
    from raggedroute_b200.ep import plan
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=G)
    try:
        xs, wr, we = _problem()
        x = xs[rank]
        local = E // G
        logits = oracle.chain_logits_f32(x, wr)
        ids, w = oracle.top2_f32(logits)
        counts = oracle.histogram(ids, E)
        offsets = oracle.exclusive_scan(counts)
        xp, pos, _, _ = oracle.stable_permute(x, ids, offsets, E, 2)
        gathered = [torch.zeros(E, dtype=torch.int32) for _ in range(G)]
        dist.all_gather(gathered, torch.from_numpy(counts))
        count_all = torch.stack(gathered).numpy()
        send_rows, send_off, recv_rows, recv_off = plan(count_all, rank)
        recv = torch.zeros(int(recv_rows.sum()), K)
        dist.all_to_all_single(recv, torch.from_numpy(xp), [int(v) for v in recv_rows],
                               [int(v) for v in send_rows])
        # Expert GEMM per (source, local expert) group, weight set = group % local.
        yr = np.zeros((recv.shape[0], N), np.float64)
        row = 0
        for p in range(G):
            for le in range(local):
                c = int(count_all[p, rank * local + le])
                yr[row:row + c] = recv[row:row + c].numpy().astype(np.float64) @ \
                    we[rank * local + le].astype(np.float64)
                row += c
        yp = torch.zeros(2 * T, N, dtype=torch.float64)
        dist.all_to_all_single(yp, torch.from_numpy(yr), [int(v) for v in send_rows],
                               [int(v) for v in recv_rows])
        y = oracle.unpermute_f64(yp.numpy().astype(np.float32), pos, w)
        np.save(os.path.join(out_dir, f"y{rank}.npy"), y)
    finally:
        dist.destroy_process_group()


def test_ep_two_rank_gloo_matches_single_process(tmp_path, rrlib, oracle):
    port = _free_port()
    mp.start_processes(_ep_worker, args=(port, str(tmp_path)), nprocs=G, join=True,
                       start_method="spawn")
    xs, wr, we = _problem()
    for rank in range(G):
        logits = oracle.chain_logits_f32(xs[rank], wr)
        ids, w = oracle.top2_f32(logits)
        counts = oracle.histogram(ids, E)
        offsets = oracle.exclusive_scan(counts)
        xp, pos, _, _ = oracle.stable_permute(xs[rank], ids, offsets, E, 2)
        yp = oracle.grouped_gemm_f64(xp, we, offsets).astype(np.float32)
        ref = oracle.unpermute_f64(yp, pos, w)
        got = np.load(tmp_path / f"y{rank}.npy")
        np.testing.assert_allclose(got, ref, rtol=1e-6, atol=1e-6)


def test_replicated_placement_splits_hot_experts():
    from raggedroute_b200.placement import ReplicatedPlacement
    rng = np.random.default_rng(0)
    e = 128
    from raggedroute_b200.workloads import zipf_log_bias
    logits = rng.standard_normal((20000, e)) + zipf_log_bias(e, 1.0)[None, :]
    loads = np.bincount(np.argsort(-logits, axis=1)[:, :2].reshape(-1), minlength=e)
    for g in (1, 2, 4, 8):
        pl = ReplicatedPlacement(loads, g)
        v = pl.virtual_experts
        assert v % g == 0 and v <= 1024
        # Every source rank maps every real expert to a virtual copy of it.
        for s in range(g):
            assert np.array_equal(pl.virtual_to_real[pl.remap[s]], np.arange(e))
        # Replicas of one expert sit on distinct ranks.
        local = v // g
        for r_e in np.flatnonzero(pl.replicas > 1):
            vids = {int(pl.remap[s, r_e]) for s in range(g)}
            assert len({vid // local for vid in vids}) == len(vids)
        assert pl.imbalance() < 1.05, (g, pl.imbalance())
    # Without skew nothing is replicated.
    flat = ReplicatedPlacement(np.ones(64), 8)
    assert flat.virtual_experts == 64 and flat.imbalance() == 1.0
