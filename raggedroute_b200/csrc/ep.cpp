// Expert-parallel chain_from_tokens (one process per GPU).
//
// The reference is single-GPU. Here the chain shards by expert. The router
// scores R real experts; the gate rewrites each selected real id through a
// per-rank remap table into one of V "virtual" experts, and rank g owns the
// contiguous virtual range [g*L, (g+1)*L), L = V / nranks. A virtual expert
// is a real expert's weights placed on one rank; a hot expert gets several
// virtual copies on different ranks and each source rank's remap sends its
// tokens to one of them (raggedroute_b200/placement.py builds the tables).
//
// Peer transport (one node; every rank maps every other rank's buffers
// through CUDA IPC at create time). Per step, on the caller's stream:
//   1. local: router GEMM, biased top-2 gate with remap, histogram+scan;
//   2. ncclAllGather of the V counts; a one-CTA kernel turns them into
//      dest_off (where this rank's rows of each expert start on the owner)
//      and the owner's grouped-GEMM offsets. Receive buffers are
//      expert-major: local expert, then source rank;
//   3. the permute kernel copies every route's row once, from x straight into
//      the owner's receive buffer (a peer store over NVLink), together with
//      its return address (source rank, permuted slot);
//   4. barrier (one-word ncclAllReduce): all rows have landed;
//   5. grouped GEMM over the receive buffer; its epilogue stores each output
//      row at its return address in the source rank's y buffer;
//   6. barrier: all outputs have landed; local unpermute.
// With RAGGEDROUTE_B200_EP_DISPATCH_SMS=n (n > 0) steps 3-5 overlap the
// dispatch with the GEMM: the owners' local experts are split
// in halves; the first half is dispatched and barriered, then its GEMM runs
// on all SMs but a few while the second half is dispatched from those few
// SMs on a second stream (a copy kernel that takes its positions from the
// route_pos the permute wrote), and after a barrier the second half's GEMM
// runs.
// No host synchronisation inside a step; the next call (or
// rr_ep_last_step_rows) waits for the previous step with a deadline. The
// barriers also order steps: a rank's next dispatch cannot start before every
// owner's GEMM of the current step ended, and no owner writes outputs before
// every source finished reading the previous ones.
//
// NCCL transport (any topology):
//   2'. ncclAllGather of the counts; one pinned read of the G x V counts
//      (the only host synchronisation) gives every rank its NCCL sizes;
//   3'. the rows this rank routed to its own experts go straight into the
//      grouped GEMM (x_permuted -> y_permuted, no copy);
//   4'. the other G-1 blocks move in G-1 pairwise rounds on a communication
//      stream (round i: send to rank+i, receive from rank-i); the grouped GEMM
//      of a received block (one group per local expert, weight set = local
//      expert) starts as soon as its round lands;
//   5'. combine: after a block's GEMM its y rows go back in the matching
//      reverse round, landing where the x rows came from in x_permuted;
//   6'. local unpermute once every combine round has landed.
// The communicator is non-blocking; every host wait on NCCL or the stream has
// a deadline, after which the communicator is aborted and RR_COMM_ERROR is
// returned, so a lost peer cannot hang the caller forever; before the abort a
// host-set fence tells every kernel still queued to store nothing into
// other ranks' memory (peer transport). Plan-time
// allocation only: receive buffers are sized for the worst case
// (nranks * 2 * max_tokens rows).
#include <cuda_runtime.h>
#include <nccl.h>

#include <atomic>
#include <chrono>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <new>
#include <thread>
#include <vector>

#include "../../include/raggedroute_b200.h"
#include "common.cuh"

struct rr_ep {
  ncclComm_t comm = nullptr;
  int nranks = 1;
  int rank = 0;
  int experts = 0;         // virtual experts (routing metadata, exchange)
  int router_experts = 0;  // real experts scored by the router
  int local = 0;
  int max_tokens = 0;
  int hidden = 0;
  int output = 0;
  double timeout_s = 60.0;
  long long capacity_rows = 0;
  float* recv_x = nullptr;
  float* recv_y = nullptr;
  int32_t* count_all = nullptr;
  int32_t* recv_offsets = nullptr;
  int32_t* h_count_all = nullptr;  // pinned
  cudaStream_t comm_stream = nullptr;
  cudaEvent_t local_ready = nullptr;
  cudaEvent_t combine_done = nullptr;
  std::vector<cudaEvent_t> dispatched;  // per round
  std::vector<cudaEvent_t> computed;    // per round
  bool broken = false;
  long long last_sent = 0;
  long long last_received = 0;
  // Peer transport.
  int transport = RR_EP_TRANSPORT_NCCL;
  int64_t* recv_ret = nullptr;     // [capacity] return address of each received row
  float* y_back = nullptr;         // [2 * max_tokens, output] outputs of this rank's routes
  int32_t* dest_off = nullptr;     // [experts]
  int32_t* barrier_word = nullptr;
  unsigned* d_err = nullptr;       // capacity overflow flag of the step
  float** d_x_base = nullptr;      // [nranks] every rank's recv_x in this address space
  int64_t** d_ret_base = nullptr;  // [nranks] every rank's recv_ret
  float** d_y_base = nullptr;      // [nranks] every rank's y_back
  std::vector<void*> imported;     // IPC mappings to close
  // Dispatch/GEMM overlap (peer transport): SMs given to the second half's
  // dispatch while the first half's grouped GEMM runs (0 = no overlap), and
  // the events that order the dispatch stream (comm_stream) against the
  // caller's.
  int overlap_sms = 0;
  cudaEvent_t half0_ready = nullptr;
  cudaEvent_t half1_sent = nullptr;
  // Step bookkeeping in two slots, so that a call only waits for the step
  // before the previous one and the host keeps one step queued ahead.
  unsigned* h_err = nullptr;        // pinned [2]
  int32_t* h_recv_total = nullptr;  // pinned [2]
  cudaEvent_t step_done[2] = {nullptr, nullptr};
  // Abort fence: host memory mapped into the device, set before the
  // communicator is aborted. Kernels of a step that was already queued
  // behind a collective that the abort ends read it and then store nothing
  // into other ranks' memory (a lost rank's buffers may be gone).
  volatile int* h_abort = nullptr;
  int* d_abort = nullptr;
  bool step_pending[2] = {false, false};
  long long step_sent[2] = {0, 0};
  int next_slot = 0;
};

namespace {

// SMs the second half's dispatch runs on beside the first half's grouped
// GEMM (peer transport); 0 = no overlap. Off by default: at 2 GPUs the split
// measured slower (10.92 ms/step with 8 SMs, 11.22 with 16, against 10.52
// without), the first half's GEMM losing more to the SMs it gives up than
// the hidden half of the dispatch saves.
constexpr int kDefaultOverlapSms = 0;

rr_status st(int32_t code, const char* msg, int32_t cuda_err = 0) {
  rr_status s;
  s.code = code;
  s.cuda_error = cuda_err;
  s.message = msg;
  return s;
}

rr_status ok() { return st(RR_SUCCESS, "success"); }

using Clock = std::chrono::steady_clock;

// Raises the abort fence, then aborts the communicator.
void abort_comm(rr_ep* ep) {
  ep->broken = true;
  if (ep->h_abort != nullptr) {
    *ep->h_abort = 1;
    std::atomic_thread_fence(std::memory_order_seq_cst);
  }
  if (ep->comm != nullptr) ncclCommAbort(ep->comm);
  ep->comm = nullptr;
}

// Waits until a non-blocking communicator leaves ncclInProgress.
rr_status wait_comm(rr_ep* ep, const char* what) {
  const auto deadline = Clock::now() + std::chrono::duration<double>(ep->timeout_s);
  while (true) {
    ncclResult_t async = ncclSuccess;
    const ncclResult_t r = ncclCommGetAsyncError(ep->comm, &async);
    if (r != ncclSuccess || (async != ncclSuccess && async != ncclInProgress)) {
      abort_comm(ep);
      return st(RR_COMM_ERROR, what);
    }
    if (async == ncclSuccess) return ok();
    if (Clock::now() > deadline) {
      abort_comm(ep);
      return st(RR_COMM_ERROR, "NCCL did not finish before the deadline; communicator aborted");
    }
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
}

rr_status check_nccl(rr_ep* ep, ncclResult_t r, const char* what) {
  if (r == ncclSuccess) return ok();
  if (r == ncclInProgress) return wait_comm(ep, what);
  abort_comm(ep);
  return st(RR_COMM_ERROR, what);
}

// Waits for all work on `stream` with a deadline, watching the communicator.
rr_status wait_stream(rr_ep* ep, cudaStream_t stream) {
  const auto deadline = Clock::now() + std::chrono::duration<double>(ep->timeout_s);
  while (true) {
    const cudaError_t q = cudaStreamQuery(stream);
    if (q == cudaSuccess) return ok();
    if (q != cudaErrorNotReady) return st(RR_CUDA_ERROR, "stream failed during EP step", q);
    if (ep->comm != nullptr) {
      ncclResult_t async = ncclSuccess;
      ncclCommGetAsyncError(ep->comm, &async);
      if (async != ncclSuccess && async != ncclInProgress) {
        abort_comm(ep);
        return st(RR_COMM_ERROR, "NCCL reported an asynchronous error");
      }
    }
    if (Clock::now() > deadline) {
      abort_comm(ep);
      return st(RR_COMM_ERROR, "EP step did not finish before the deadline; communicator aborted");
    }
    std::this_thread::sleep_for(std::chrono::microseconds(10));
  }
}

void free_ep(rr_ep* ep) {
  if (ep == nullptr) return;
  for (void* p : ep->imported) cudaIpcCloseMemHandle(p);
  ep->imported.clear();
  cudaFree(ep->recv_ret);
  cudaFree(ep->y_back);
  cudaFree(ep->dest_off);
  cudaFree(ep->barrier_word);
  cudaFree(ep->d_err);
  cudaFree(ep->d_x_base);
  cudaFree(ep->d_ret_base);
  cudaFree(ep->d_y_base);
  cudaFreeHost(ep->h_err);
  if (ep->h_abort != nullptr) cudaFreeHost(const_cast<int*>(ep->h_abort));
  cudaFreeHost(ep->h_recv_total);
  for (cudaEvent_t ev : ep->step_done) {
    if (ev != nullptr) cudaEventDestroy(ev);
  }
  cudaFree(ep->recv_x);
  cudaFree(ep->recv_y);
  cudaFree(ep->count_all);
  cudaFree(ep->recv_offsets);
  cudaFreeHost(ep->h_count_all);
  for (cudaEvent_t ev : ep->dispatched) cudaEventDestroy(ev);
  for (cudaEvent_t ev : ep->computed) cudaEventDestroy(ev);
  if (ep->local_ready != nullptr) cudaEventDestroy(ep->local_ready);
  if (ep->half0_ready != nullptr) cudaEventDestroy(ep->half0_ready);
  if (ep->half1_sent != nullptr) cudaEventDestroy(ep->half1_sent);
  if (ep->combine_done != nullptr) cudaEventDestroy(ep->combine_done);
  if (ep->comm_stream != nullptr) cudaStreamDestroy(ep->comm_stream);
  if (ep->comm != nullptr) ncclCommDestroy(ep->comm);
  delete ep;
}

// Waits for `ev` with the plan's deadline, watching the communicator.
rr_status wait_event(rr_ep* ep, cudaEvent_t ev) {
  const auto deadline = Clock::now() + std::chrono::duration<double>(ep->timeout_s);
  while (true) {
    const cudaError_t q = cudaEventQuery(ev);
    if (q == cudaSuccess) return ok();
    if (q != cudaErrorNotReady) return st(RR_CUDA_ERROR, "EP step failed on the device", q);
    if (ep->comm != nullptr) {
      ncclResult_t async = ncclSuccess;
      ncclCommGetAsyncError(ep->comm, &async);
      if (async != ncclSuccess && async != ncclInProgress) {
        abort_comm(ep);
        return st(RR_COMM_ERROR, "NCCL reported an asynchronous error");
      }
    }
    if (Clock::now() > deadline) {
      abort_comm(ep);
      return st(RR_COMM_ERROR, "EP step did not finish before the deadline; communicator aborted");
    }
    std::this_thread::sleep_for(std::chrono::microseconds(10));
  }
}

// One-word all-reduce used as a cross-rank barrier in stream order.
rr_status barrier(rr_ep* ep, cudaStream_t stream) {
  return check_nccl(ep, ncclAllReduce(ep->barrier_word, ep->barrier_word, 1, ncclInt32, ncclMax,
                                      ep->comm, stream),
                    "NCCL barrier failed");
}

// Completes the bookkeeping of the peer-transport step that used `slot`.
rr_status finish_slot(rr_ep* ep, int slot) {
  if (!ep->step_pending[slot]) return ok();
  const rr_status s = wait_event(ep, ep->step_done[slot]);
  if (s.code != RR_SUCCESS) return s;
  ep->step_pending[slot] = false;
  ep->last_sent = ep->step_sent[slot];
  ep->last_received = ep->h_recv_total[slot];
  if (ep->h_err[slot] != 0) {
    ep->h_err[slot] = 0;
    cudaMemset(ep->d_err, 0, sizeof(unsigned));
    return st(RR_INSUFFICIENT_WORKSPACE,
              "a rank received more rows than its receive capacity (tokens above max_tokens)");
  }
  return ok();
}

// Completes every outstanding step, oldest first.
rr_status finish_all(rr_ep* ep) {
  const int older = ep->next_slot;  // the slot used two calls ago
  rr_status s = finish_slot(ep, older);
  const rr_status t = finish_slot(ep, older ^ 1);
  return s.code != RR_SUCCESS ? s : t;
}

// All ranks agree on a flag (minimum over ranks). Collective.
rr_status agree(rr_ep* ep, int32_t* d_flag, int mine, bool* all) {
  cudaStream_t s = ep->comm_stream;
  int32_t h = mine;
  cudaError_t e = cudaMemcpyAsync(d_flag, &h, sizeof(h), cudaMemcpyHostToDevice, s);
  if (e != cudaSuccess) return st(RR_CUDA_ERROR, "EP flag upload failed", e);
  rr_status r = check_nccl(ep, ncclAllReduce(d_flag, d_flag, 1, ncclInt32, ncclMin, ep->comm, s),
                           "NCCL agreement failed");
  if (r.code != RR_SUCCESS) return r;
  e = cudaMemcpyAsync(&h, d_flag, sizeof(h), cudaMemcpyDeviceToHost, s);
  if (e != cudaSuccess) return st(RR_CUDA_ERROR, "EP flag read-back failed", e);
  r = wait_stream(ep, s);
  if (r.code != RR_SUCCESS) return r;
  *all = h != 0;
  return ok();
}

void release_peer(rr_ep* ep) {
  for (void* p : ep->imported) cudaIpcCloseMemHandle(p);
  ep->imported.clear();
  cudaFree(ep->recv_ret);
  cudaFree(ep->y_back);
  cudaFree(ep->d_x_base);
  cudaFree(ep->d_ret_base);
  cudaFree(ep->d_y_base);
  ep->recv_ret = nullptr;
  ep->y_back = nullptr;
  ep->d_x_base = nullptr;
  ep->d_ret_base = nullptr;
  ep->d_y_base = nullptr;
  cudaGetLastError();
}

// Maps every rank's recv_x, recv_ret and y_back into this process (CUDA IPC
// handles exchanged with ncclAllGather). Collective; every rank reaches the
// same verdict. *mapped is false when some rank could not take part.
rr_status setup_peer(rr_ep* ep, bool* mapped) {
  *mapped = false;
  const int G = ep->nranks;
  cudaStream_t s = ep->comm_stream;
  constexpr int kSlot = 4 * static_cast<int>(sizeof(cudaIpcMemHandle_t));
  uint8_t* d_slots = nullptr;
  int32_t* d_flag = nullptr;
  cudaError_t e = cudaMalloc(&d_slots, static_cast<std::size_t>(kSlot) * G);
  if (e == cudaSuccess) e = cudaMalloc(&d_flag, sizeof(int32_t));
  if (e != cudaSuccess) {
    cudaFree(d_slots);
    cudaGetLastError();
    return st(RR_CUDA_ERROR, "EP peer setup: device allocation failed", e);
  }
  // Local part: buffers and their handles. A failure here is reported
  // through the exchange so that every rank takes the same branch.
  int local_ok = 1;
  if (cudaMalloc(&ep->recv_ret, sizeof(int64_t) * ep->capacity_rows) != cudaSuccess ||
      cudaMalloc(&ep->y_back, sizeof(float) * 2LL * ep->max_tokens * ep->output) !=
          cudaSuccess ||
      cudaMalloc(&ep->d_x_base, sizeof(float*) * G) != cudaSuccess ||
      cudaMalloc(&ep->d_ret_base, sizeof(int64_t*) * G) != cudaSuccess ||
      cudaMalloc(&ep->d_y_base, sizeof(float*) * G) != cudaSuccess) {
    local_ok = 0;
    cudaGetLastError();
  }
  // Rows never written hold an out-of-range address and are skipped.
  if (local_ok && cudaMemset(ep->recv_ret, 0xff, sizeof(int64_t) * ep->capacity_rows) !=
                      cudaSuccess) {
    local_ok = 0;
    cudaGetLastError();
  }
  std::vector<uint8_t> slots(static_cast<std::size_t>(kSlot) * G, 0);
  uint8_t* mine = slots.data() + static_cast<std::size_t>(kSlot) * ep->rank;
  if (local_ok) {
    cudaIpcMemHandle_t h[3];
    if (cudaIpcGetMemHandle(&h[0], ep->recv_x) != cudaSuccess ||
        cudaIpcGetMemHandle(&h[1], ep->recv_ret) != cudaSuccess ||
        cudaIpcGetMemHandle(&h[2], ep->y_back) != cudaSuccess) {
      local_ok = 0;
      cudaGetLastError();
    } else {
      std::memcpy(mine, h, sizeof(h));
    }
  }
  mine[kSlot - 1] = static_cast<uint8_t>(local_ok);
  rr_status r = ok();
  e = cudaMemcpyAsync(d_slots + static_cast<std::size_t>(kSlot) * ep->rank, mine, kSlot,
                      cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) {
    r = check_nccl(ep, ncclAllGather(d_slots + static_cast<std::size_t>(kSlot) * ep->rank,
                                     d_slots, kSlot, ncclUint8, ep->comm, s),
                   "NCCL exchange of memory handles failed");
    if (r.code == RR_SUCCESS) {
      e = cudaMemcpyAsync(slots.data(), d_slots, slots.size(), cudaMemcpyDeviceToHost, s);
      if (e == cudaSuccess) r = wait_stream(ep, s);
    }
  }
  if (e != cudaSuccess) r = st(RR_CUDA_ERROR, "EP peer setup: handle exchange failed", e);
  bool all = r.code == RR_SUCCESS;
  for (int p = 0; all && p < G; ++p) all = slots[static_cast<std::size_t>(kSlot) * p + kSlot - 1] != 0;
  // Open every peer's buffers.
  std::vector<float*> xb(G), yb(G);
  std::vector<int64_t*> rb(G);
  int open_ok = all ? 1 : 0;
  for (int p = 0; open_ok && p < G; ++p) {
    if (p == ep->rank) {
      xb[p] = ep->recv_x;
      rb[p] = ep->recv_ret;
      yb[p] = ep->y_back;
      continue;
    }
    cudaIpcMemHandle_t h[3];
    std::memcpy(h, slots.data() + static_cast<std::size_t>(kSlot) * p, sizeof(h));
    void* ptr[3] = {nullptr, nullptr, nullptr};
    for (int i = 0; i < 3 && open_ok; ++i) {
      if (cudaIpcOpenMemHandle(&ptr[i], h[i], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
        open_ok = 0;
        cudaGetLastError();
      } else {
        ep->imported.push_back(ptr[i]);
      }
    }
    xb[p] = static_cast<float*>(ptr[0]);
    rb[p] = static_cast<int64_t*>(ptr[1]);
    yb[p] = static_cast<float*>(ptr[2]);
  }
  if (r.code == RR_SUCCESS) {
    r = agree(ep, d_flag, open_ok, &all);
  }
  cudaFree(d_slots);
  cudaFree(d_flag);
  if (r.code != RR_SUCCESS) return r;
  if (!all) {
    release_peer(ep);
    return ok();
  }
  e = cudaMemcpy(ep->d_x_base, xb.data(), sizeof(float*) * G, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) {
    e = cudaMemcpy(ep->d_ret_base, rb.data(), sizeof(int64_t*) * G, cudaMemcpyHostToDevice);
  }
  if (e == cudaSuccess) {
    e = cudaMemcpy(ep->d_y_base, yb.data(), sizeof(float*) * G, cudaMemcpyHostToDevice);
  }
  if (e != cudaSuccess) return st(RR_CUDA_ERROR, "EP peer setup: pointer tables failed", e);
  *mapped = true;
  return ok();
}

}  // namespace

extern "C" {

rr_status rr_ep_get_unique_id(void* unique_id) {
  if (unique_id == nullptr) return st(RR_INVALID_ARGUMENT, "unique_id must not be null");
  static_assert(sizeof(ncclUniqueId) == RR_EP_UNIQUE_ID_BYTES, "unique id size");
  ncclUniqueId id;
  if (ncclGetUniqueId(&id) != ncclSuccess) return st(RR_COMM_ERROR, "ncclGetUniqueId failed");
  std::memcpy(unique_id, &id, sizeof(id));
  return ok();
}

// Pure host arithmetic of one rank's exchange, exposed for tests and tools.
// count_all: [nranks][experts] per-source expert counts. Outputs (nranks
// entries each): rows this rank sends to / receives from every peer and the
// row offsets of those blocks in x_permuted / the receive buffer.
rr_status rr_ep_plan(const int32_t* count_all, int nranks, int rank, int experts,
                     int64_t* send_rows, int64_t* send_offsets, int64_t* recv_rows,
                     int64_t* recv_offsets) {
  if (count_all == nullptr || send_rows == nullptr || send_offsets == nullptr ||
      recv_rows == nullptr || recv_offsets == nullptr) {
    return st(RR_INVALID_ARGUMENT, "rr_ep_plan received a null pointer");
  }
  if (nranks < 1 || rank < 0 || rank >= nranks || experts < nranks || experts % nranks != 0) {
    return st(RR_INVALID_ARGUMENT, "rr_ep_plan requires experts to be a multiple of nranks");
  }
  const int local = experts / nranks;
  int64_t so = 0, ro = 0;
  for (int p = 0; p < nranks; ++p) {
    int64_t s = 0, r = 0;
    for (int le = 0; le < local; ++le) {
      s += count_all[static_cast<int64_t>(rank) * experts + p * local + le];
      r += count_all[static_cast<int64_t>(p) * experts + rank * local + le];
    }
    send_rows[p] = s;
    send_offsets[p] = so;
    recv_rows[p] = r;
    recv_offsets[p] = ro;
    so += s;
    ro += r;
  }
  return ok();
}

rr_status rr_ep_create(const void* unique_id, int nranks, int rank, int router_experts,
                       int experts, int max_tokens, int hidden, int output,
                       double timeout_seconds, int transport, rr_ep** out) {
  if (out == nullptr) return st(RR_INVALID_ARGUMENT, "out must not be null");
  *out = nullptr;
  if (nranks < 1 || rank < 0 || rank >= nranks || experts < 2 || experts > RR_MAX_EXPERTS ||
      experts % nranks != 0 || router_experts < 2 || router_experts > RR_MAX_EXPERTS ||
      max_tokens <= 0 || hidden <= 0 || output <= 0 ||
      static_cast<long long>(nranks) * 2 * max_tokens > 0x7fffffffLL) {
    return st(RR_INVALID_ARGUMENT,
              "rr_ep_create requires nranks | virtual experts <= 1024, positive sizes and "
              "nranks * 2 * max_tokens < 2^31");
  }
  if (transport != RR_EP_TRANSPORT_AUTO && transport != RR_EP_TRANSPORT_NCCL &&
      transport != RR_EP_TRANSPORT_PEER) {
    return st(RR_INVALID_ARGUMENT, "unknown EP transport");
  }
  if (nranks > 1 && unique_id == nullptr) {
    return st(RR_INVALID_ARGUMENT, "unique_id must not be null for nranks > 1");
  }
  rr_ep* ep = new (std::nothrow) rr_ep();
  if (ep == nullptr) return st(RR_INVALID_ARGUMENT, "out of host memory");
  ep->nranks = nranks;
  ep->rank = rank;
  ep->experts = experts;
  ep->router_experts = router_experts;
  ep->local = experts / nranks;
  ep->max_tokens = max_tokens;
  ep->hidden = hidden;
  ep->output = output;
  ep->timeout_s = timeout_seconds > 0 ? timeout_seconds : 60.0;
  ep->capacity_rows = static_cast<long long>(nranks) * 2 * max_tokens;
  cudaError_t e = cudaSuccess;
  if (nranks > 1) e = cudaMalloc(&ep->recv_x, sizeof(float) * ep->capacity_rows * hidden);
  if (e == cudaSuccess) e = cudaMalloc(&ep->count_all, sizeof(int32_t) * nranks * experts);
  if (e == cudaSuccess) e = cudaMalloc(&ep->recv_offsets, sizeof(int32_t) * (experts + 1));
  if (e == cudaSuccess) e = cudaMalloc(&ep->dest_off, sizeof(int32_t) * experts);
  if (e == cudaSuccess) e = cudaMalloc(&ep->barrier_word, sizeof(int32_t));
  if (e == cudaSuccess) e = cudaMemset(ep->barrier_word, 0, sizeof(int32_t));
  if (e == cudaSuccess) e = cudaMalloc(&ep->d_err, sizeof(unsigned));
  if (e == cudaSuccess) e = cudaMemset(ep->d_err, 0, sizeof(unsigned));
  if (e == cudaSuccess) e = cudaMallocHost(&ep->h_count_all, sizeof(int32_t) * nranks * experts);
  if (e == cudaSuccess) e = cudaMallocHost(&ep->h_err, 2 * sizeof(unsigned));
  if (e == cudaSuccess) e = cudaMallocHost(&ep->h_recv_total, 2 * sizeof(int32_t));
  if (e == cudaSuccess) {
    void* h = nullptr;
    e = cudaHostAlloc(&h, sizeof(int), cudaHostAllocMapped);
    if (e == cudaSuccess) {
      ep->h_abort = static_cast<volatile int*>(h);
      *ep->h_abort = 0;
      e = cudaHostGetDevicePointer(reinterpret_cast<void**>(&ep->d_abort), h, 0);
    }
  }
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&ep->comm_stream, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ep->local_ready, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ep->combine_done, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ep->half0_ready, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ep->half1_sent, cudaEventDisableTiming);
  {
    // Every rank must use the same setting (it changes the sequence of
    // collectives): the variable is read once here.
    const char* v = std::getenv("RAGGEDROUTE_B200_EP_DISPATCH_SMS");
    ep->overlap_sms = v != nullptr ? std::atoi(v) : kDefaultOverlapSms;
    if (ep->overlap_sms < 0) ep->overlap_sms = 0;
    ep->overlap_sms = (ep->overlap_sms + 1) & ~1;  // whole CTA pairs
  }
  for (int i = 0; e == cudaSuccess && i < 2; ++i) {
    e = cudaEventCreateWithFlags(&ep->step_done[i], cudaEventDisableTiming);
  }
  for (int i = 0; e == cudaSuccess && i < nranks; ++i) {
    cudaEvent_t a = nullptr, b = nullptr;
    e = cudaEventCreateWithFlags(&a, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&b, cudaEventDisableTiming);
    ep->dispatched.push_back(a);
    ep->computed.push_back(b);
  }
  if (e != cudaSuccess) {
    cudaGetLastError();
    free_ep(ep);
    return st(RR_CUDA_ERROR, "rr_ep_create: device allocation failed", e);
  }
  ep->h_err[0] = ep->h_err[1] = 0;
  ep->h_recv_total[0] = ep->h_recv_total[1] = 0;
  if (nranks > 1) {
    ncclUniqueId id;
    std::memcpy(&id, unique_id, sizeof(id));
    ncclConfig_t config = NCCL_CONFIG_INITIALIZER;
    config.blocking = 0;
    const ncclResult_t r = ncclCommInitRankConfig(&ep->comm, nranks, id, rank, &config);
    if (r != ncclSuccess && r != ncclInProgress) {
      free_ep(ep);
      return st(RR_COMM_ERROR, "ncclCommInitRankConfig failed");
    }
    const rr_status w = wait_comm(ep, "NCCL communicator initialisation failed");
    if (w.code != RR_SUCCESS) {
      free_ep(ep);
      return w;
    }
    bool mapped = false;
    if (transport != RR_EP_TRANSPORT_NCCL) {
      const rr_status p = setup_peer(ep, &mapped);
      if (p.code != RR_SUCCESS) {
        free_ep(ep);
        return p;
      }
      if (!mapped && transport == RR_EP_TRANSPORT_PEER) {
        free_ep(ep);
        return st(RR_COMM_ERROR, "the peer transport needs every rank to map every other rank's "
                                 "memory (CUDA IPC over NVLink); use the NCCL transport");
      }
    }
    ep->transport = mapped ? RR_EP_TRANSPORT_PEER : RR_EP_TRANSPORT_NCCL;
    if (!mapped) {
      e = cudaMalloc(&ep->recv_y, sizeof(float) * ep->capacity_rows * output);
      if (e != cudaSuccess) {
        cudaGetLastError();
        free_ep(ep);
        return st(RR_CUDA_ERROR, "rr_ep_create: device allocation failed", e);
      }
    }
  } else {
    ep->transport = transport == RR_EP_TRANSPORT_PEER ? RR_EP_TRANSPORT_PEER
                                                      : RR_EP_TRANSPORT_NCCL;
  }
  *out = ep;
  return ok();
}

rr_status rr_ep_destroy(rr_ep* ep) {
  if (ep == nullptr) return ok();
  rr_status s = finish_all(ep);
  // Other ranks may still write into this rank's buffers until they pass a
  // barrier placed after their last step.
  if (ep->nranks > 1 && ep->comm != nullptr && ep->transport == RR_EP_TRANSPORT_PEER) {
    const rr_status b = barrier(ep, ep->comm_stream);
    if (b.code == RR_SUCCESS) {
      const rr_status w = wait_stream(ep, ep->comm_stream);
      if (s.code == RR_SUCCESS) s = w;
    } else if (s.code == RR_SUCCESS) {
      s = b;
    }
  }
  free_ep(ep);
  return s;
}

rr_status rr_ep_transport(const rr_ep* ep, int* transport) {
  if (ep == nullptr || transport == nullptr) {
    return st(RR_INVALID_ARGUMENT, "ep and transport must not be null");
  }
  *transport = ep->transport;
  return ok();
}

rr_status rr_ep_last_step_rows(const rr_ep* ep, int64_t* rows_sent, int64_t* rows_received) {
  if (ep == nullptr) return st(RR_INVALID_ARGUMENT, "ep must not be null");
  const rr_status s = finish_all(const_cast<rr_ep*>(ep));
  if (s.code != RR_SUCCESS) return s;
  if (rows_sent != nullptr) *rows_sent = ep->last_sent;
  if (rows_received != nullptr) *rows_received = ep->last_received;
  return ok();
}

rr_status rr_ep_chain_from_tokens(rr_ep* ep, const float* x, const float* router_weights,
                                  const float* logit_bias, const int32_t* expert_remap,
                                  const float* local_expert_weights,
                                  float* logits, int32_t* expert_ids, float* route_weights,
                                  int32_t* counts, int32_t* offsets, float* x_permuted,
                                  int32_t* route_pos, float* y_permuted, float* y, int tokens,
                                  const rr_context* ctx) {
  if (ep == nullptr || ctx == nullptr) return st(RR_INVALID_ARGUMENT, "ep and ctx are required");
  if (ep->broken) return st(RR_COMM_ERROR, "the EP communicator was aborted earlier");
  {
    const rr_status prev = finish_slot(ep, ep->next_slot);
    if (prev.code != RR_SUCCESS) return prev;
  }
  const bool peer = ep->nranks > 1 && ep->transport == RR_EP_TRANSPORT_PEER;
  if (tokens < 0 || tokens > ep->max_tokens) {
    return st(RR_INVALID_ARGUMENT, "tokens must be in [0, max_tokens] of the EP plan");
  }
  const int E = ep->experts, K = ep->hidden, N = ep->output, G = ep->nranks;
  const int RE = ep->router_experts;
  if (expert_remap == nullptr && RE != E) {
    return st(RR_INVALID_ARGUMENT, "an expert remap is required when virtual != router experts");
  }
  // A rank with no tokens still takes part in the exchange (its experts
  // receive rows); its token-indexed buffers may then be NULL.
  const bool need_rows = tokens > 0;
  if (router_weights == nullptr || local_expert_weights == nullptr || counts == nullptr ||
      offsets == nullptr ||
      (need_rows && (x == nullptr || logits == nullptr || expert_ids == nullptr ||
                     route_weights == nullptr || route_pos == nullptr || y == nullptr)) ||
      (!peer && need_rows && (x_permuted == nullptr || y_permuted == nullptr))) {
    return st(RR_INVALID_ARGUMENT, "rr_ep_chain_from_tokens received a null device buffer");
  }
  const std::size_t need = rrb::permute_workspace_bytes(tokens, E, 2);
  if (ctx->workspace == nullptr || ctx->workspace_bytes < need) {
    return st(RR_INSUFFICIENT_WORKSPACE, "EP chain requires rr_chain_workspace_size bytes");
  }
  cudaStream_t stream = static_cast<cudaStream_t>(ctx->stream);
  const int routes = 2 * tokens;
  // 1. Local stages (identical to the single-GPU chain).
  cudaError_t e = cudaSuccess;
  if (tokens > 0) {
    e = rrb::launch_grouped_gemm(x, router_weights, nullptr, logits, 1, tokens, K, RE, stream);
    if (e == cudaSuccess) {
      e = rrb::launch_topk_gate(logits, logit_bias, expert_ids, route_weights, tokens, RE, stream,
                                expert_remap);
    }
  }
  if (e == cudaSuccess) {
    e = rrb::launch_histogram_exclusive_scan(expert_ids, counts, offsets, routes, E, stream);
  }
  if (e == cudaSuccess && tokens > 0 && !peer) {
    e = rrb::launch_token_permute(x, expert_ids, offsets, x_permuted, route_pos, nullptr, tokens,
                                  E, 2, K, ctx->workspace, stream);
  }
  if (e != cudaSuccess) return st(RR_CUDA_ERROR, "EP local stage launch failed", e);

  if (peer) {
    // 2. Counts exchange and the receive layout, on the device.
    rr_status s = check_nccl(
        ep, ncclAllGather(counts, ep->count_all, E, ncclInt32, ep->comm, stream),
        "ncclAllGather of expert counts failed");
    if (s.code != RR_SUCCESS) return s;
    e = rrb::launch_ep_peer_layout(ep->count_all, ep->dest_off, ep->recv_offsets, G, E, ep->rank,
                                   ep->local, ep->capacity_rows, ep->d_err, stream);
    // 3. Dispatch fused into the permute. With the overlap (every rank makes
    // the same choice: it depends on the plan only) the owners' local
    // experts are split in two halves: the first half's rows go out on all
    // SMs; then, while the first half's grouped GEMM runs on all SMs but
    // overlap_sms, the second half's rows go out from a persistent dispatch
    // on those SMs (on comm_stream); the second half's GEMM follows once
    // every rank's second half has landed. No kernel waits on another: the
    // two halves meet only at NCCL barriers on the caller's stream. The
    // permute places (and ranks) every route; it sends only the first half.
    const int L = ep->local;
    const bool split = ep->overlap_sms > 0 && L >= 2 && 4 * ep->overlap_sms < rrb::sm_count();
    const int half = split ? L / 2 : L;
    rrb::PeerDispatch pd;
    pd.x_base = ep->d_x_base;
    pd.ret_base = ep->d_ret_base;
    pd.dest_off = ep->dest_off;
    pd.local = L;
    pd.me = ep->rank;
    pd.capacity = ep->capacity_rows;
    pd.err = ep->d_err;
    pd.abort = ep->d_abort;
    pd.le_lo = 0;
    pd.le_hi = half;
    if (e == cudaSuccess && tokens > 0) {
      e = rrb::launch_token_permute_peer(x, expert_ids, offsets, route_pos, tokens, E, 2, K,
                                         ctx->workspace, pd, stream);
    }
    if (e != cudaSuccess) return st(RR_CUDA_ERROR, "EP dispatch launch failed", e);
    // 4. Every rank's rows (of the first half) have landed.
    s = barrier(ep, stream);
    if (s.code != RR_SUCCESS) return s;
    // 5. Expert GEMM over the receive buffer, combine fused into its epilogue.
    rrb::RowScatter sc;
    sc.dst = ep->recv_ret;
    sc.base = ep->d_y_base;
    sc.nranks = G;
    sc.row_limit = 2LL * ep->max_tokens;
    sc.abort = ep->d_abort;
    if (split) {
      e = cudaEventRecord(ep->half0_ready, stream);
      if (e == cudaSuccess) e = cudaStreamWaitEvent(ep->comm_stream, ep->half0_ready, 0);
      if (e == cudaSuccess && tokens > 0) {
        pd.le_lo = half;
        pd.le_hi = L;
        e = rrb::launch_ep_dispatch_rest(x, expert_ids, offsets, route_pos, tokens, E, 2, K, pd,
                                         ep->overlap_sms, ep->comm_stream);
      }
      if (e == cudaSuccess) e = cudaEventRecord(ep->half1_sent, ep->comm_stream);
      if (e != cudaSuccess) return st(RR_CUDA_ERROR, "EP second-half dispatch launch failed", e);
      // The first half's GEMM walks a static tile schedule, so all of its
      // CTA pairs must be resident beside the dispatch (which takes whole
      // SM pairs, so every GPC keeps an even number of free SMs).
      rrb::RowScatter sc0 = sc;
      sc0.max_ctas = rrb::sm_count() - ep->overlap_sms;
      e = rrb::launch_grouped_gemm(ep->recv_x, local_expert_weights, ep->recv_offsets,
                                   ep->y_back, half, static_cast<int>(ep->capacity_rows), K, N,
                                   stream, 0, &sc0);
      if (e == cudaSuccess) e = cudaStreamWaitEvent(stream, ep->half1_sent, 0);
      if (e != cudaSuccess) return st(RR_CUDA_ERROR, "EP grouped GEMM launch failed", e);
      // Every rank's second half has landed.
      s = barrier(ep, stream);
      if (s.code != RR_SUCCESS) return s;
      e = rrb::launch_grouped_gemm(ep->recv_x,
                                   local_expert_weights + static_cast<long long>(half) * K * N,
                                   ep->recv_offsets + half, ep->y_back, L - half,
                                   static_cast<int>(ep->capacity_rows), K, N, stream, 0, &sc);
    } else {
      e = rrb::launch_grouped_gemm(ep->recv_x, local_expert_weights, ep->recv_offsets,
                                   ep->y_back, L, static_cast<int>(ep->capacity_rows), K, N,
                                   stream, 0, &sc);
    }
    if (e != cudaSuccess) return st(RR_CUDA_ERROR, "EP grouped GEMM launch failed", e);
    // 6. Every rank's outputs have landed; local unpermute.
    s = barrier(ep, stream);
    if (s.code != RR_SUCCESS) return s;
    if (tokens > 0) {
      e = rrb::launch_unpermute(ep->y_back, route_pos, route_weights, y, tokens, 2, N, stream);
      if (e != cudaSuccess) return st(RR_CUDA_ERROR, "EP unpermute launch failed", e);
    }
    const int slot = ep->next_slot;
    e = cudaMemcpyAsync(ep->h_recv_total + slot, ep->recv_offsets + ep->local, sizeof(int32_t),
                        cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess) {
      e = cudaMemcpyAsync(ep->h_err + slot, ep->d_err, sizeof(unsigned), cudaMemcpyDeviceToHost,
                          stream);
    }
    if (e == cudaSuccess) e = cudaEventRecord(ep->step_done[slot], stream);
    if (e != cudaSuccess) return st(RR_CUDA_ERROR, "EP step bookkeeping failed", e);
    ep->step_pending[slot] = true;
    ep->step_sent[slot] = routes;
    ep->next_slot = slot ^ 1;
    return ok();
  }

  if (G == 1) {
    if (tokens > 0) {
      e = rrb::launch_grouped_gemm(x_permuted, local_expert_weights, offsets, y_permuted, E,
                                   routes, K, N, stream);
      if (e == cudaSuccess) {
        e = rrb::launch_unpermute(y_permuted, route_pos, route_weights, y, tokens, 2, N, stream);
      }
    }
    ep->last_sent = ep->last_received = routes;
    return e == cudaSuccess ? ok() : st(RR_CUDA_ERROR, "EP launch failed", e);
  }

  // 2. Counts exchange and the step's exchange plan (all NCCL work runs on
  //    the communication stream, in the same order on every rank).
  cudaStream_t cs = ep->comm_stream;
  e = cudaEventRecord(ep->local_ready, stream);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(cs, ep->local_ready, 0);
  if (e != cudaSuccess) return st(RR_CUDA_ERROR, "EP stream ordering failed", e);
  rr_status s = check_nccl(ep, ncclAllGather(counts, ep->count_all, E, ncclInt32, ep->comm, cs),
                           "ncclAllGather of expert counts failed");
  if (s.code != RR_SUCCESS) return s;
  e = cudaMemcpyAsync(ep->h_count_all, ep->count_all, sizeof(int32_t) * G * E,
                      cudaMemcpyDeviceToHost, cs);
  if (e != cudaSuccess) return st(RR_CUDA_ERROR, "counts read-back failed", e);
  s = wait_stream(ep, cs);
  if (s.code != RR_SUCCESS) return s;
  std::vector<int64_t> send_rows(G), send_off(G), recv_rows(G), recv_off(G);
  s = rr_ep_plan(ep->h_count_all, G, ep->rank, E, send_rows.data(), send_off.data(),
                 recv_rows.data(), recv_off.data());
  if (s.code != RR_SUCCESS) return s;
  ep->last_sent = send_off[G - 1] + send_rows[G - 1];
  ep->last_received = recv_off[G - 1] + recv_rows[G - 1];
  e = rrb::launch_ep_recv_offsets(ep->count_all, ep->recv_offsets, G, E, ep->rank, ep->local,
                                  stream);
  if (e != cudaSuccess) return st(RR_CUDA_ERROR, "receive offsets launch failed", e);

  const int g = ep->rank;
  const int L = ep->local;
  // 3. This rank's own block: no transfer.
  if (send_rows[g] > 0) {
    e = rrb::launch_grouped_gemm(x_permuted, local_expert_weights, offsets + g * L, y_permuted, L,
                                 routes, K, N, stream, L);
    if (e != cudaSuccess) return st(RR_CUDA_ERROR, "EP grouped GEMM launch failed", e);
  }
  // 4. Dispatch rounds; each received block's GEMM waits for its round.
  for (int i = 1; i < G; ++i) {
    const int dst = (g + i) % G;
    const int src = (g - i + G) % G;
    ncclGroupStart();
    if (send_rows[dst] > 0) {
      ncclSend(x_permuted + send_off[dst] * K, static_cast<size_t>(send_rows[dst]) * K, ncclFloat,
               dst, ep->comm, cs);
    }
    if (recv_rows[src] > 0) {
      ncclRecv(ep->recv_x + recv_off[src] * K, static_cast<size_t>(recv_rows[src]) * K, ncclFloat,
               src, ep->comm, cs);
    }
    s = check_nccl(ep, ncclGroupEnd(), "NCCL dispatch failed");
    if (s.code != RR_SUCCESS) return s;
    e = cudaEventRecord(ep->dispatched[i], cs);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(stream, ep->dispatched[i], 0);
    if (e == cudaSuccess && recv_rows[src] > 0) {
      e = rrb::launch_grouped_gemm(ep->recv_x, local_expert_weights, ep->recv_offsets + src * L,
                                   ep->recv_y, L, static_cast<int>(ep->last_received), K, N,
                                   stream, L);
    }
    if (e == cudaSuccess) e = cudaEventRecord(ep->computed[i], stream);
    if (e != cudaSuccess) return st(RR_CUDA_ERROR, "EP dispatch/GEMM ordering failed", e);
  }
  // 5. Combine rounds: block i returns to its source as soon as its GEMM ends.
  for (int i = 1; i < G; ++i) {
    const int dst = (g + i) % G;
    const int src = (g - i + G) % G;
    e = cudaStreamWaitEvent(cs, ep->computed[i], 0);
    if (e != cudaSuccess) return st(RR_CUDA_ERROR, "EP combine ordering failed", e);
    ncclGroupStart();
    if (recv_rows[src] > 0) {
      ncclSend(ep->recv_y + recv_off[src] * N, static_cast<size_t>(recv_rows[src]) * N, ncclFloat,
               src, ep->comm, cs);
    }
    if (send_rows[dst] > 0) {
      ncclRecv(y_permuted + send_off[dst] * N, static_cast<size_t>(send_rows[dst]) * N, ncclFloat,
               dst, ep->comm, cs);
    }
    s = check_nccl(ep, ncclGroupEnd(), "NCCL combine failed");
    if (s.code != RR_SUCCESS) return s;
  }
  e = cudaEventRecord(ep->combine_done, cs);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(stream, ep->combine_done, 0);
  if (e != cudaSuccess) return st(RR_CUDA_ERROR, "EP combine ordering failed", e);

  // 6. Local unpermute.
  if (tokens > 0) {
    e = rrb::launch_unpermute(y_permuted, route_pos, route_weights, y, tokens, 2, N, stream);
    if (e != cudaSuccess) return st(RR_CUDA_ERROR, "EP unpermute launch failed", e);
  }
  return ok();
}

}  // extern "C"
