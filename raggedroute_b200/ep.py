"""Python handle for the expert-parallel runtime (rr_ep_* in the C ABI).

torch.distributed is only the bootstrap here: rank 0 asks the library for an
NCCL unique id and the process group broadcasts it; the library then owns
its own NCCL communicator and does every exchange itself.
"""
from __future__ import annotations

import ctypes
import dataclasses

import torch
import torch.distributed as dist

from raggedroute_b200._lib import Context, check, lib
from raggedroute_b200.ops import ChainBuffers, _ctx, _ptr

UNIQUE_ID_BYTES = 128
TRANSPORTS = {"auto": 0, "nccl": 1, "peer": 2}


class ExpertParallel:
    """`experts` virtual experts (V) are split evenly over the ranks; the
    router scores `router_experts` real experts (R, default V) and
    chain_from_tokens takes this rank's remap table R -> V when they differ.
    transport: "auto" (peer memory when every rank maps every other rank's
    buffers, else NCCL), "peer" or "nccl"; `self.transport` is the one used."""

    def __init__(self, experts: int, max_tokens: int, hidden: int, output: int,
                 rank: int | None = None, world: int | None = None, group=None,
                 timeout_s: float = 120.0, router_experts: int | None = None,
                 transport: str = "auto"):
        self.rank = dist.get_rank(group) if rank is None else rank
        self.world = dist.get_world_size(group) if world is None else world
        self.experts, self.hidden, self.output = experts, hidden, output
        self.router_experts = experts if router_experts is None else router_experts
        self.local = experts // self.world
        uid = torch.zeros(UNIQUE_ID_BYTES, dtype=torch.uint8)
        if self.world > 1:
            if self.rank == 0:
                buf = (ctypes.c_uint8 * UNIQUE_ID_BYTES)()
                check(lib().rr_ep_get_unique_id(ctypes.cast(buf, ctypes.c_void_p)),
                      "rr_ep_get_unique_id")
                uid = torch.tensor(list(buf), dtype=torch.uint8)
            dev_uid = uid.cuda() if dist.get_backend(group) == "nccl" else uid
            dist.broadcast(dev_uid, src=0, group=group)
            uid = dev_uid.cpu()
        raw = (ctypes.c_uint8 * UNIQUE_ID_BYTES)(*uid.tolist())
        handle = ctypes.c_void_p()
        check(lib().rr_ep_create(ctypes.cast(raw, ctypes.c_void_p), self.world, self.rank,
                                 self.router_experts, experts, max_tokens, hidden, output,
                                 timeout_s, TRANSPORTS[transport], ctypes.byref(handle)),
              "rr_ep_create")
        self._h = handle
        t = ctypes.c_int()
        check(lib().rr_ep_transport(self._h, ctypes.byref(t)), "rr_ep_transport")
        self.transport = {v: k for k, v in TRANSPORTS.items()}[t.value]

    def chain_from_tokens(self, x: torch.Tensor, router_weights: torch.Tensor,
                          local_expert_weights: torch.Tensor, buf: ChainBuffers,
                          logit_bias: torch.Tensor | None = None,
                          expert_remap: torch.Tensor | None = None,
                          ctx: Context | None = None) -> torch.Tensor:
        """buf must be allocated for V virtual experts with logits [T, R]. The
        peer transport leaves buf.x_permuted / buf.y_permuted unwritten."""
        tokens = x.shape[0]
        check(lib().rr_ep_chain_from_tokens(
            self._h, _ptr(x), _ptr(router_weights), _ptr(logit_bias), _ptr(expert_remap),
            _ptr(local_expert_weights),
            _ptr(buf.logits), _ptr(buf.expert_ids), _ptr(buf.route_weights), _ptr(buf.counts),
            _ptr(buf.offsets), _ptr(buf.x_permuted), _ptr(buf.route_pos), _ptr(buf.y_permuted),
            _ptr(buf.y), tokens, _ctx(ctx, buf.workspace)), "rr_ep_chain_from_tokens")
        return buf.y

    def last_step_rows(self) -> tuple[int, int]:
        s, r = ctypes.c_int64(), ctypes.c_int64()
        check(lib().rr_ep_last_step_rows(self._h, ctypes.byref(s), ctypes.byref(r)),
              "rr_ep_last_step_rows")
        return int(s.value), int(r.value)

    def close(self) -> None:
        if self._h:
            lib().rr_ep_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass


class HostPipeline:
    """ExpertParallel.chain_from_tokens over host memory, pipelined across
    calls: X is copied in on one copy stream into one of two device slots,
    the step runs on ctx.stream, and Y is copied out on another copy stream
    from one of two output slots. A call's copy in waits only for the step two
    calls back to have finished reading its slot, so it overlaps the previous
    step's compute and copy out (x_host must be complete when the call is
    made, as with RR_HOST_CHAIN_INPUT_READY). Completion, Y in y_host
    included, is ordered on ctx.stream. All other chain buffers are shared
    between the slots: they are used only on ctx.stream, in call order.
    x_host / y_host should be pinned. Y equals ExpertParallel.chain_from_tokens
    on the same tokens bit for bit."""

    def __init__(self, ep: ExpertParallel, buf: ChainBuffers, max_tokens: int, device):
        self.ep, self.buf = ep, buf
        self.x_dev = [torch.empty(max_tokens, ep.hidden, device=device) for _ in range(2)]
        self.y_dev = [torch.empty(max_tokens, ep.output, device=device) for _ in range(2)]
        self.h2d = torch.cuda.Stream(device)
        self.d2h = torch.cuda.Stream(device)
        ev = lambda: [torch.cuda.Event() for _ in range(2)]  # noqa: E731
        self.h2d_done, self.compute_done, self.d2h_done = ev(), ev(), ev()
        self.calls = 0

    def __call__(self, x_host: torch.Tensor, router_weights: torch.Tensor,
                 local_expert_weights: torch.Tensor, y_host: torch.Tensor,
                 logit_bias: torch.Tensor | None = None,
                 expert_remap: torch.Tensor | None = None,
                 ctx: Context | None = None) -> torch.Tensor:
        tokens = x_host.shape[0]
        if tokens > self.x_dev[0].shape[0]:
            raise ValueError("more tokens than the pipeline was sized for")
        slot = self.calls & 1
        first_use = self.calls < 2
        self.calls += 1
        main = torch.cuda.ExternalStream(ctx.stream) if ctx is not None and ctx.stream \
            else torch.cuda.current_stream()
        x, y = self.x_dev[slot][:tokens], self.y_dev[slot][:tokens]
        if not first_use:
            self.h2d.wait_event(self.compute_done[slot])
        with torch.cuda.stream(self.h2d):
            x.copy_(x_host, non_blocking=True)
            self.h2d_done[slot].record(self.h2d)
        main.wait_event(self.h2d_done[slot])
        if not first_use:
            main.wait_event(self.d2h_done[slot])
        buf = dataclasses.replace(self.buf, y=y)
        self.ep.chain_from_tokens(x, router_weights, local_expert_weights, buf,
                                  logit_bias=logit_bias, expert_remap=expert_remap, ctx=ctx)
        self.compute_done[slot].record(main)
        self.d2h.wait_event(self.compute_done[slot])
        with torch.cuda.stream(self.d2h):
            y_host.copy_(y, non_blocking=True)
            self.d2h_done[slot].record(self.d2h)
        main.wait_event(self.d2h_done[slot])
        return y_host


def plan(count_all, rank: int):
    """rr_ep_plan for a [nranks, experts] int32 array (host)."""
    import numpy as np
    c = np.ascontiguousarray(count_all, dtype=np.int32)
    g, e = c.shape
    out = [np.zeros(g, np.int64) for _ in range(4)]
    ptr = lambda a: a.ctypes.data_as(ctypes.c_void_p)  # noqa: E731
    check(lib().rr_ep_plan(ptr(c), g, rank, e, *[ptr(a) for a in out]), "rr_ep_plan")
    return tuple(out)  # send_rows, send_offsets, recv_rows, recv_offsets
