"""Expert-parallel chain on the GPU.

* One rank (no communicator): rr_ep_chain_from_tokens equals
  rr_chain_from_tokens bit for bit, also through HostPipeline (host memory,
  calls overlapped).
* Two or more GPUs: tests/ep_worker.py under torchrun, for both transports
  (peer memory and NCCL), with equal or ragged per-rank token counts (one
  rank idle), and for the peer transport with and without the dispatch/GEMM
  overlap; every rank's EP output must equal its single-GPU chain bit for bit
  (replicated hot experts, Zipf logit bias). Skipped, with the
  reason, when fewer than two GPUs are visible.
"""
from __future__ import annotations

import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_ep_single_rank_matches_chain(rrlib, cuda):
    from raggedroute_b200.ep import ExpertParallel
    from raggedroute_b200.workloads import normal, zipf_log_bias
    t, k, e, n = 2000, 256, 64, 128
    x = normal((t, k), 1.0, 11, cuda)
    wr = normal((k, e), 1 / 16, 12, cuda)
    we = normal((e, k, n), 1 / 16, 13, cuda)
    bias = torch.from_numpy(zipf_log_bias(e, 1.0)).to(cuda)
    ep = ExpertParallel(e, t, k, n, rank=0, world=1)
    b1 = rrlib.ChainBuffers.allocate(t, k, e, n, cuda)
    b2 = rrlib.ChainBuffers.allocate(t, k, e, n, cuda)
    ep.chain_from_tokens(x, wr, we, b1, logit_bias=bias)
    rrlib.chain_from_tokens(x, wr, we, b2, logit_bias=bias)
    torch.cuda.synchronize()
    assert torch.equal(b1.route_pos, b2.route_pos)
    assert torch.equal(b1.y.view(torch.int32), b2.y.view(torch.int32))
    assert ep.last_step_rows() == (2 * t, 2 * t)
    ep.close()


def test_ep_host_pipeline_matches_chain(rrlib, cuda):
    """HostPipeline: three batches of different sizes queued back to back
    over pinned host memory; each Y equals the device chain bit for bit."""
    from raggedroute_b200.ep import ExpertParallel, HostPipeline
    from raggedroute_b200.workloads import normal, zipf_log_bias
    t, k, e, n = 1500, 256, 64, 128
    wr = normal((k, e), 1 / 16, 12, cuda)
    we = normal((e, k, n), 1 / 16, 13, cuda)
    bias = torch.from_numpy(zipf_log_bias(e, 1.0)).to(cuda)
    ep = ExpertParallel(e, t, k, n, rank=0, world=1)
    buf = rrlib.ChainBuffers.allocate(t, k, e, n, cuda)
    stream = torch.cuda.Stream(cuda)
    ctx = rrlib.Context(stream=stream.cuda_stream)
    pipe = HostPipeline(ep, buf, t, cuda)
    xs = [normal((m, k), 1.0, 40 + m, "cpu").pin_memory() for m in (1500, 999, 1300)]
    ys = [torch.empty(x.shape[0], n).pin_memory() for x in xs]
    for x, y in zip(xs, ys):
        pipe(x, wr, we, y, logit_bias=bias, ctx=ctx)
    stream.synchronize()
    for x, y in zip(xs, ys):
        ref = rrlib.ChainBuffers.allocate(x.shape[0], k, e, n, cuda)
        rrlib.chain_from_tokens(x.to(cuda), wr, we, ref, logit_bias=bias)
        torch.cuda.synchronize()
        assert torch.equal(y.view(torch.int32), ref.y.cpu().view(torch.int32))
    ep.close()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs at least 2 GPUs")
@pytest.mark.parametrize("transport,ragged,overlap,port", [
    ("peer", "0", "8", 29531), ("peer", "1", "8", 29532), ("peer", "1", "0", 29535),
    ("nccl", "0", "8", 29533), ("nccl", "1", "8", 29534)])
def test_ep_multi_gpu_matches_single_gpu_chain(rrlib, cuda, transport, ragged, overlap, port):
    """overlap: SMs of the peer transport's second-half dispatch beside the
    first half's grouped GEMM (RAGGEDROUTE_B200_EP_DISPATCH_SMS; 0 = one
    dispatch, then one GEMM)."""
    world = min(torch.cuda.device_count(), 8)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", EP_TRANSPORT=transport, EP_RAGGED=ragged,
               RAGGEDROUTE_B200_EP_DISPATCH_SMS=overlap)
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", f"--nproc-per-node={world}", "--master-addr=127.0.0.1",
           f"--master-port={port}", os.path.join(ROOT, "tests", "ep_worker.py")]
    res = subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=ROOT)
    assert res.returncode == 0, res.stdout[-4000:] + res.stderr[-4000:]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs at least 2 GPUs")
def test_ep_lost_rank_returns_comm_error(rrlib, cuda):
    """tests/ep_fail_worker.py: a rank leaves between steps; the other's next
    step returns RR_COMM_ERROR within its deadline (no hang, no GPU fault)
    and its device stays usable. NCCL transport (no peer-memory stores),
    NVLS off, gloo bootstrap."""
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "180", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node=2", "--master-addr=127.0.0.1",
           "--master-port=29541", os.path.join(ROOT, "tests", "ep_fail_worker.py")]
    res = subprocess.run(cmd, capture_output=True, text=True, env=env, cwd=ROOT)
    out = res.stdout + res.stderr
    assert res.returncode == 0, out[-4000:]
    assert "rank 0: ok=True" in out, out[-4000:]
