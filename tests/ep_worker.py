"""Multi-GPU expert-parallel check, launched by tests/test_gpu_ep.py as
`torchrun --nproc-per-node G tests/ep_worker.py`. Every rank runs its own
token batch through rr_ep_chain_from_tokens and through the single-GPU
rr_chain_from_tokens with all experts; ids, counts, route weights and the
output must be identical bit for bit (each output row is computed by the
same kernels in the same K order wherever its expert lives).

EP_TRANSPORT selects the transport ("peer" or "nccl"; the plan must use the
one asked for). EP_RAGGED=1 gives rank r T - 997*r tokens and the last rank
none, so ranks exchange unequal blocks and an idle rank still serves its
experts."""
from __future__ import annotations

import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main() -> int:
    import raggedroute_b200 as rr
    from raggedroute_b200.ep import ExpertParallel
    from raggedroute_b200.placement import ReplicatedPlacement
    from raggedroute_b200.workloads import normal, zipf_log_bias

    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local_rank = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    t_max, k, e, n = int(os.environ.get("EP_T", "3000")), 256, 32, 96  # E % world == 0
    transport = os.environ.get("EP_TRANSPORT", "auto")
    t = t_max
    if os.environ.get("EP_RAGGED") == "1":
        t = 0 if rank == world - 1 else max(1, t_max - 997 * rank)
    x = normal((t, k), 1.0, 1000 + rank, dev)
    wr = normal((k, e), 1 / 16, 7, dev)
    we = normal((e, k, n), 1 / 16, 8, dev)
    bias = torch.from_numpy(zipf_log_bias(e, 1.0)).to(dev)
    b_ref = rr.ChainBuffers.allocate(t, k, e, n, dev)
    # Loads from this batch's routing, summed over ranks -> replicated placement.
    if t > 0:
        rr.chain_from_tokens(x, wr, we, b_ref, logit_bias=bias)
        loads = b_ref.counts.to(torch.float64)
    else:
        loads = torch.zeros(e, dtype=torch.float64, device=dev)
    dist.all_reduce(loads)
    pl = ReplicatedPlacement(loads.cpu().numpy(), world)
    v = pl.virtual_experts
    local = v // world
    v2r_all = torch.from_numpy(pl.virtual_to_real).to(dev)
    local_w = we[v2r_all[rank * local:(rank + 1) * local]].contiguous()
    remap = torch.from_numpy(pl.remap[rank]).to(dev)
    ep = ExpertParallel(v, t_max, k, n, router_experts=e, transport=transport)
    ok = transport == "auto" or ep.transport == transport
    if not ok:
        print(f"rank {rank}: asked for {transport}, plan uses {ep.transport}", flush=True)
    b_ep = rr.ChainBuffers.allocate(t, k, v, n, dev, router_experts=e)
    for step in range(3):
        ep.chain_from_tokens(x, wr, local_w, b_ep, logit_bias=bias, expert_remap=remap)
        if t == 0:
            torch.cuda.synchronize()
            continue
        rr.chain_from_tokens(x, wr, we, b_ref, logit_bias=bias)
        torch.cuda.synchronize()
        # Virtual ids map back to the single-GPU chain's real ids; virtual
        # counts sum to the real counts.
        if not torch.equal(v2r_all[b_ep.expert_ids.long()].to(torch.int32), b_ref.expert_ids):
            print(f"rank {rank} step {step}: expert ids differ", flush=True)
            ok = False
        real_counts = torch.zeros(e, dtype=torch.int64, device=dev)
        real_counts.index_add_(0, v2r_all, b_ep.counts.to(torch.int64))
        if not torch.equal(real_counts.to(torch.int32), b_ref.counts):
            print(f"rank {rank} step {step}: counts differ", flush=True)
            ok = False
        if not torch.equal(b_ep.route_weights, b_ref.route_weights):
            print(f"rank {rank} step {step}: route weights differ", flush=True)
            ok = False
        if not torch.equal(b_ep.y.view(torch.int32), b_ref.y.view(torch.int32)):
            diff = (b_ep.y - b_ref.y).abs().max().item()
            print(f"rank {rank} step {step}: y differs (max {diff})", flush=True)
            ok = False
    sent, received = ep.last_step_rows()
    rows = torch.tensor([sent, received], dtype=torch.int64, device=dev)
    dist.all_reduce(rows)
    if sent != 2 * t or rows[0].item() != rows[1].item():
        print(f"rank {rank}: rows sent {sent}, totals {rows.tolist()}", flush=True)
        ok = False
    flag = torch.tensor([1 if ok else 0], device=dev)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    ep.close()
    dist.destroy_process_group()
    print(f"rank {rank}: transport={ep.transport} ok={ok} sent={sent} received={received}",
          flush=True)
    return 0 if int(flag.item()) == 1 else 1


if __name__ == "__main__":
    sys.exit(main())
