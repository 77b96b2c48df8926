"""Multi-GPU expert-parallel check, launched by tests/test_gpu_ep.py as
`torchrun --nproc-per-node G tests/ep_worker.py`. Every rank runs its own
token batch through rr_ep_chain_from_tokens and through the single-GPU
rr_chain_from_tokens with all experts; ids, counts, offsets, route_pos and
the output must be identical bit for bit (each output row is computed by the
same kernels in the same K order wherever its expert lives)."""
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
    from raggedroute_b200.placement import (expected_loads_from_bias, lpt_placement,
                                            relabel_permutation)
    from raggedroute_b200.workloads import normal, zipf_log_bias

    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local_rank = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    t, k, e, n = int(os.environ.get("EP_T", "3000")), 256, 32, 96
    x = normal((t, k), 1.0, 1000 + rank, dev)
    wr = normal((k, e), 1 / 16, 7, dev)
    we = normal((e, k, n), 1 / 16, 8, dev)
    bias_np = zipf_log_bias(e, 1.0)
    perm = relabel_permutation(lpt_placement(expected_loads_from_bias(bias_np), world))
    perm_t = torch.from_numpy(perm).to(dev)
    wr = wr[:, perm_t].contiguous()
    we = we[perm_t].contiguous()
    bias = torch.from_numpy(bias_np[perm]).to(dev)
    local = e // world
    local_w = we[rank * local:(rank + 1) * local].contiguous()

    ep = ExpertParallel(e, t, k, n)
    b_ep = rr.ChainBuffers.allocate(t, k, e, n, dev)
    b_ref = rr.ChainBuffers.allocate(t, k, e, n, dev)
    ok = True
    for step in range(2):
        ep.chain_from_tokens(x, wr, local_w, b_ep, logit_bias=bias)
        rr.chain_from_tokens(x, wr, we, b_ref, logit_bias=bias)
        torch.cuda.synchronize()
        for name in ("expert_ids", "counts", "offsets", "route_pos"):
            if not torch.equal(getattr(b_ep, name), getattr(b_ref, name)):
                print(f"rank {rank} step {step}: {name} differs", flush=True)
                ok = False
        if not torch.equal(b_ep.y.view(torch.int32), b_ref.y.view(torch.int32)):
            diff = (b_ep.y - b_ref.y).abs().max().item()
            print(f"rank {rank} step {step}: y differs (max {diff})", flush=True)
            ok = False
    sent, received = ep.last_step_rows()
    flag = torch.tensor([1 if ok else 0], device=dev)
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    ep.close()
    dist.destroy_process_group()
    print(f"rank {rank}: ok={ok} sent={sent} received={received}", flush=True)
    return 0 if int(flag.item()) == 1 else 1


if __name__ == "__main__":
    sys.exit(main())
