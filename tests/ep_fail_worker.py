"""Expert-parallel failure detection, launched by tests/test_gpu_ep.py as
`torchrun --nproc-per-node 2 tests/ep_fail_worker.py` (gloo bootstrap, NCCL
transport inside the library, NVLS off). Both ranks run one EP step; rank 1
then leaves between steps (all its work finished) without destroying its
plan. Rank 0's next step must come back with RR_COMM_ERROR within a few
times its 3 s deadline (the communicator is aborted, never a hang), later
calls on the plan must fail fast, and the device must stay usable: a
single-GPU chain right after is exact against a chain run before."""
from __future__ import annotations

import datetime
import os
import sys
import time

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main() -> int:
    import raggedroute_b200 as rr
    from raggedroute_b200._lib import RaggedRouteError, StatusCode
    from raggedroute_b200.ep import ExpertParallel
    from raggedroute_b200.workloads import normal

    rank = int(os.environ["RANK"])
    local_rank = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    t, k, e, n = 1024, 128, 16, 64
    x = normal((t, k), 1.0, 100 + rank, dev)
    wr = normal((k, e), 1 / 16, 7, dev)
    we = normal((e, k, n), 1 / 16, 8, dev)
    local = e // 2
    ep = ExpertParallel(e, t, k, n, timeout_s=3.0, transport="nccl")
    buf = rr.ChainBuffers.allocate(t, k, e, n, dev)
    ep.chain_from_tokens(x, wr, we[rank * local:(rank + 1) * local].contiguous(), buf)
    ep.last_step_rows()  # waits for the step on this rank
    torch.cuda.synchronize()
    ref = rr.ChainBuffers.allocate(t, k, e, n, dev)
    rr.chain_from_tokens(x, wr, we, ref)
    torch.cuda.synchronize()
    y_before = ref.y.clone()
    dist.barrier()  # both ranks finished step 1
    if rank == 1:
        os._exit(0)  # leaves between steps, plan not destroyed
    t0 = time.monotonic()
    code = None
    try:
        ep.chain_from_tokens(x, wr, we[:local].contiguous(), buf)
        ep.last_step_rows()
    except RaggedRouteError as exc:
        code = exc.code
    waited = time.monotonic() - t0
    ok = code == StatusCode.COMM_ERROR and waited < 30.0
    print(f"rank 0: step after peer loss -> {code} in {waited:.1f} s", flush=True)
    t1 = time.monotonic()
    try:
        ep.chain_from_tokens(x, wr, we[:local].contiguous(), buf)
        ok = False
    except RaggedRouteError as exc:
        ok = ok and exc.code == StatusCode.COMM_ERROR and time.monotonic() - t1 < 1.0
    ep.close()
    rr.chain_from_tokens(x, wr, we, ref)
    torch.cuda.synchronize()
    ok = ok and torch.equal(ref.y.view(torch.int32), y_before.view(torch.int32))
    print(f"rank 0: ok={ok}", flush=True)
    os._exit(0 if ok else 1)


if __name__ == "__main__":
    sys.exit(main())
