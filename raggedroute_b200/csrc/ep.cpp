// Expert-parallel chain_from_tokens over NCCL (one process per GPU).
//
// The reference is single-GPU. Here the chain shards by expert. The router
// scores R real experts; the gate rewrites each selected real id through a
// per-rank remap table into one of V "virtual" experts, and rank g owns the
// contiguous virtual range [g*L, (g+1)*L), L = V / nranks. A virtual expert
// is a real expert's weights placed on one rank; a hot expert gets several
// virtual copies on different ranks and each source rank's remap sends its
// tokens to one of them (raggedroute_b200/placement.py builds the tables).
// Per step, on the caller's stream:
//   1. local: router GEMM, biased top-2 gate, histogram+scan over all E,
//      stable permute -> rows for rank p are contiguous in x_permuted;
//   2. ncclAllGather of the E counts; one pinned read of the G x E counts
//      (the only host synchronisation) gives every rank its NCCL sizes;
//   3. the rows this rank routed to its own experts go straight into the
//      grouped GEMM (x_permuted -> y_permuted, no copy);
//   4. the other G-1 blocks move in G-1 pairwise rounds on a communication
//      stream (round i: send to rank+i, receive from rank-i); the grouped GEMM
//      of a received block (one group per local expert, weight set = local
//      expert) starts as soon as its round lands, so transfers overlap the
//      GEMM of earlier blocks;
//   5. combine: after a block's GEMM its y rows go back in the matching
//      reverse round, landing where the x rows came from in x_permuted;
//   6. local unpermute once every combine round has landed.
// The communicator is non-blocking; every host wait on NCCL or the stream has
// a deadline, after which the communicator is aborted and RR_COMM_ERROR is
// returned, so a lost peer cannot hang the caller forever. Plan-time
// allocation only: receive buffers are sized for the worst case
// (nranks * 2 * max_tokens rows).
#include <cuda_runtime.h>
#include <nccl.h>

#include <chrono>
#include <cstdint>
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
};

namespace {

rr_status st(int32_t code, const char* msg, int32_t cuda_err = 0) {
  rr_status s;
  s.code = code;
  s.cuda_error = cuda_err;
  s.message = msg;
  return s;
}

rr_status ok() { return st(RR_SUCCESS, "success"); }

using Clock = std::chrono::steady_clock;

// Waits until a non-blocking communicator leaves ncclInProgress.
rr_status wait_comm(rr_ep* ep, const char* what) {
  const auto deadline = Clock::now() + std::chrono::duration<double>(ep->timeout_s);
  while (true) {
    ncclResult_t async = ncclSuccess;
    const ncclResult_t r = ncclCommGetAsyncError(ep->comm, &async);
    if (r != ncclSuccess || (async != ncclSuccess && async != ncclInProgress)) {
      ep->broken = true;
      ncclCommAbort(ep->comm);
      ep->comm = nullptr;
      return st(RR_COMM_ERROR, what);
    }
    if (async == ncclSuccess) return ok();
    if (Clock::now() > deadline) {
      ep->broken = true;
      ncclCommAbort(ep->comm);
      ep->comm = nullptr;
      return st(RR_COMM_ERROR, "NCCL did not finish before the deadline; communicator aborted");
    }
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
}

rr_status check_nccl(rr_ep* ep, ncclResult_t r, const char* what) {
  if (r == ncclSuccess) return ok();
  if (r == ncclInProgress) return wait_comm(ep, what);
  ep->broken = true;
  ncclCommAbort(ep->comm);
  ep->comm = nullptr;
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
        ep->broken = true;
        ncclCommAbort(ep->comm);
        ep->comm = nullptr;
        return st(RR_COMM_ERROR, "NCCL reported an asynchronous error");
      }
    }
    if (Clock::now() > deadline) {
      ep->broken = true;
      if (ep->comm != nullptr) ncclCommAbort(ep->comm);
      ep->comm = nullptr;
      return st(RR_COMM_ERROR, "EP step did not finish before the deadline; communicator aborted");
    }
    std::this_thread::sleep_for(std::chrono::microseconds(10));
  }
}

void free_ep(rr_ep* ep) {
  if (ep == nullptr) return;
  cudaFree(ep->recv_x);
  cudaFree(ep->recv_y);
  cudaFree(ep->count_all);
  cudaFree(ep->recv_offsets);
  cudaFreeHost(ep->h_count_all);
  for (cudaEvent_t ev : ep->dispatched) cudaEventDestroy(ev);
  for (cudaEvent_t ev : ep->computed) cudaEventDestroy(ev);
  if (ep->local_ready != nullptr) cudaEventDestroy(ep->local_ready);
  if (ep->combine_done != nullptr) cudaEventDestroy(ep->combine_done);
  if (ep->comm_stream != nullptr) cudaStreamDestroy(ep->comm_stream);
  if (ep->comm != nullptr) ncclCommDestroy(ep->comm);
  delete ep;
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
                       double timeout_seconds, rr_ep** out) {
  if (out == nullptr) return st(RR_INVALID_ARGUMENT, "out must not be null");
  *out = nullptr;
  if (nranks < 1 || rank < 0 || rank >= nranks || experts < 2 || experts > RR_MAX_EXPERTS ||
      experts % nranks != 0 || router_experts < 2 || router_experts > RR_MAX_EXPERTS ||
      max_tokens <= 0 || hidden <= 0 || output <= 0 || max_tokens > (1 << 30) / 2) {
    return st(RR_INVALID_ARGUMENT,
              "rr_ep_create requires nranks | virtual experts <= 1024 and positive sizes");
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
  if (nranks > 1) {
    e = cudaMalloc(&ep->recv_x, sizeof(float) * ep->capacity_rows * hidden);
    if (e == cudaSuccess) e = cudaMalloc(&ep->recv_y, sizeof(float) * ep->capacity_rows * output);
  }
  if (e == cudaSuccess) e = cudaMalloc(&ep->count_all, sizeof(int32_t) * nranks * experts);
  if (e == cudaSuccess) e = cudaMalloc(&ep->recv_offsets, sizeof(int32_t) * (experts + 1));
  if (e == cudaSuccess) e = cudaMallocHost(&ep->h_count_all, sizeof(int32_t) * nranks * experts);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&ep->comm_stream, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ep->local_ready, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ep->combine_done, cudaEventDisableTiming);
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
  }
  *out = ep;
  return ok();
}

rr_status rr_ep_destroy(rr_ep* ep) {
  free_ep(ep);
  return ok();
}

rr_status rr_ep_last_step_rows(const rr_ep* ep, int64_t* rows_sent, int64_t* rows_received) {
  if (ep == nullptr) return st(RR_INVALID_ARGUMENT, "ep must not be null");
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
  if (tokens < 0 || tokens > ep->max_tokens) {
    return st(RR_INVALID_ARGUMENT, "tokens must be in [0, max_tokens] of the EP plan");
  }
  const int E = ep->experts, K = ep->hidden, N = ep->output, G = ep->nranks;
  const int RE = ep->router_experts;
  if (expert_remap == nullptr && RE != E) {
    return st(RR_INVALID_ARGUMENT, "an expert remap is required when virtual != router experts");
  }
  if (x == nullptr || router_weights == nullptr || local_expert_weights == nullptr ||
      logits == nullptr || expert_ids == nullptr || route_weights == nullptr ||
      counts == nullptr || offsets == nullptr || x_permuted == nullptr || route_pos == nullptr ||
      y_permuted == nullptr || y == nullptr) {
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
  if (e == cudaSuccess && tokens > 0) {
    e = rrb::launch_token_permute(x, expert_ids, offsets, x_permuted, route_pos, nullptr, tokens,
                                  E, 2, K, ctx->workspace, stream);
  }
  if (e != cudaSuccess) return st(RR_CUDA_ERROR, "EP local stage launch failed", e);

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
