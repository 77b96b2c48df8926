// chain_from_tokens over host memory, pipelined through the copy engines.
//
// The reference's chain takes device buffers (benchmarks/adapters/
// chain_adapter.cpp:263-467); a caller whose tokens live in host memory
// would copy X in, run the chain and copy Y out, one after the other. Here the
// token batch is cut into chunks that flow through three streams:
//
//   h2d stream:   X chunk c  host -> device slot c%2
//   ctx->stream:  chain_from_tokens on slot c%2 (all seven stages)
//   d2h stream:   Y chunk c  device slot c%2 -> host
//
// so the host-to-device copy of chunk c+1 and the device-to-host copy of
// chunk c-1 run on the copy engines while chunk c computes. Equal chunks: a
// tail cut into halves down to an eighth of a chunk measured slower at C5
// (2.93 against 3.01 M tokens/s), since every chunk's chain reads all active
// experts' weights whatever its size. Two device slots;
// events order reuse (a slot's X is not overwritten before the chain that
// read it ended, its Y not before the copy that read it ended). Every token's
// output depends only on its own row, its routing and the expert weights,
// and each output row is computed by the same kernels in the same K order in
// any chunk (the router GEMM takes the same kernel at every row count), so Y
// is bit-identical to one chain over the whole batch.
#include <cuda_runtime.h>

#include <cstdint>
#include <new>

#include "../../include/raggedroute_b200.h"
#include "common.cuh"

struct rr_host_chain {
  int chunk = 0;
  int hidden = 0;
  int experts = 0;
  int output = 0;
  int device = 0;
  uint32_t flags = 0;
  void* slab[2] = {nullptr, nullptr};
  std::size_t workspace_bytes = 0;
  struct Slot {
    float* x;
    float* logits;
    int32_t* ids;
    float* weights;
    int32_t* counts;
    int32_t* offsets;
    float* x_permuted;
    int32_t* route_pos;
    float* y_permuted;
    float* y;
    void* workspace;
  } slot[2] = {};
  cudaStream_t h2d = nullptr;
  cudaStream_t d2h = nullptr;
  cudaEvent_t entry = nullptr;
  cudaEvent_t h2d_done[2] = {nullptr, nullptr};
  cudaEvent_t compute_done[2] = {nullptr, nullptr};
  cudaEvent_t d2h_done[2] = {nullptr, nullptr};
};

namespace {

rr_status st(int32_t code, const char* msg, int32_t cuda_err = 0) {
  rr_status s;
  s.code = code;
  s.cuda_error = cuda_err;
  s.message = msg;
  return s;
}

std::size_t up256(std::size_t v) { return (v + 255) & ~static_cast<std::size_t>(255); }

// Carves one slot's buffers out of a slab; returns the slab size when
// base == nullptr.
std::size_t carve(rr_host_chain* p, char* base, rr_host_chain::Slot* s) {
  const std::size_t c = static_cast<std::size_t>(p->chunk);
  const std::size_t k = p->hidden, e = p->experts, n = p->output;
  const std::size_t sizes[11] = {4 * c * k,     4 * c * e, 8 * c,     8 * c,
                                 4 * e,         4 * (e + 1), 8 * c * k, 8 * c,
                                 8 * c * n,     4 * c * n, p->workspace_bytes};
  void* ptrs[11];
  std::size_t off = 0;
  for (int i = 0; i < 11; ++i) {
    ptrs[i] = base != nullptr ? base + off : nullptr;
    off += up256(sizes[i] > 0 ? sizes[i] : 1);
  }
  if (s != nullptr) {
    s->x = static_cast<float*>(ptrs[0]);
    s->logits = static_cast<float*>(ptrs[1]);
    s->ids = static_cast<int32_t*>(ptrs[2]);
    s->weights = static_cast<float*>(ptrs[3]);
    s->counts = static_cast<int32_t*>(ptrs[4]);
    s->offsets = static_cast<int32_t*>(ptrs[5]);
    s->x_permuted = static_cast<float*>(ptrs[6]);
    s->route_pos = static_cast<int32_t*>(ptrs[7]);
    s->y_permuted = static_cast<float*>(ptrs[8]);
    s->y = static_cast<float*>(ptrs[9]);
    s->workspace = ptrs[10];
  }
  return off;
}

void free_plan(rr_host_chain* p) {
  if (p == nullptr) return;
  for (int i = 0; i < 2; ++i) {
    cudaFree(p->slab[i]);
    if (p->h2d_done[i] != nullptr) cudaEventDestroy(p->h2d_done[i]);
    if (p->compute_done[i] != nullptr) cudaEventDestroy(p->compute_done[i]);
    if (p->d2h_done[i] != nullptr) cudaEventDestroy(p->d2h_done[i]);
  }
  if (p->entry != nullptr) cudaEventDestroy(p->entry);
  if (p->h2d != nullptr) cudaStreamDestroy(p->h2d);
  if (p->d2h != nullptr) cudaStreamDestroy(p->d2h);
  delete p;
}

}  // namespace

extern "C" {

rr_status rr_host_chain_create(int chunk_tokens, int hidden, int experts, int output,
                               rr_host_chain** out) {
  if (out == nullptr) return st(RR_INVALID_ARGUMENT, "out must not be null");
  *out = nullptr;
  if (chunk_tokens <= 0 || hidden <= 0 || experts < 2 || experts > RR_MAX_EXPERTS ||
      output <= 0 || chunk_tokens > (1 << 29)) {
    return st(RR_INVALID_ARGUMENT,
              "rr_host_chain_create requires positive sizes and 2 <= experts <= 1024");
  }
  rr_host_chain* p = new (std::nothrow) rr_host_chain();
  if (p == nullptr) return st(RR_INVALID_ARGUMENT, "out of host memory");
  p->chunk = chunk_tokens;
  p->hidden = hidden;
  p->experts = experts;
  p->output = output;
  p->workspace_bytes = rr_chain_workspace_size(chunk_tokens, hidden, experts, output);
  cudaError_t e = cudaGetDevice(&p->device);
  const std::size_t bytes = carve(p, nullptr, nullptr);
  for (int i = 0; e == cudaSuccess && i < 2; ++i) {
    e = cudaMalloc(&p->slab[i], bytes);
    if (e == cudaSuccess) carve(p, static_cast<char*>(p->slab[i]), &p->slot[i]);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p->h2d_done[i], cudaEventDisableTiming);
    if (e == cudaSuccess) {
      e = cudaEventCreateWithFlags(&p->compute_done[i], cudaEventDisableTiming);
    }
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p->d2h_done[i], cudaEventDisableTiming);
  }
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&p->entry, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&p->h2d, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&p->d2h, cudaStreamNonBlocking);
  if (e != cudaSuccess) {
    cudaGetLastError();
    free_plan(p);
    return st(RR_CUDA_ERROR, "rr_host_chain_create: device allocation failed", e);
  }
  *out = p;
  return st(RR_SUCCESS, "success");
}

rr_status rr_host_chain_destroy(rr_host_chain* plan) {
  if (plan != nullptr) {
    for (int i = 0; i < 2; ++i) cudaEventSynchronize(plan->d2h_done[i]);
  }
  free_plan(plan);
  return st(RR_SUCCESS, "success");
}

rr_status rr_host_chain_set_flags(rr_host_chain* plan, uint32_t flags) {
  if (plan == nullptr) return st(RR_INVALID_ARGUMENT, "plan must not be null");
  if ((flags & ~RR_HOST_CHAIN_INPUT_READY) != 0) {
    return st(RR_INVALID_ARGUMENT, "unknown host chain flag");
  }
  plan->flags = flags;
  return st(RR_SUCCESS, "success");
}

rr_status rr_chain_from_tokens_host(rr_host_chain* plan, const float* x_host,
                                    const float* router_weights, const float* logit_bias,
                                    const float* expert_weights, float* y_host,
                                    int32_t* expert_ids_host, float* route_weights_host,
                                    int tokens, const rr_context* ctx) {
  if (plan == nullptr || ctx == nullptr) {
    return st(RR_INVALID_ARGUMENT, "plan and ctx are required");
  }
  if (tokens < 0) return st(RR_INVALID_ARGUMENT, "tokens must be non-negative");
  if (tokens > 0 && (x_host == nullptr || y_host == nullptr)) {
    return st(RR_INVALID_ARGUMENT, "x_host and y_host must not be null");
  }
  if (router_weights == nullptr || expert_weights == nullptr) {
    return st(RR_INVALID_ARGUMENT, "router and expert weights must not be null");
  }
  cudaStream_t s = static_cast<cudaStream_t>(ctx->stream);
  const int K = plan->hidden, E = plan->experts, N = plan->output;
  // The call's work is ordered after the caller's earlier work on ctx->stream
  // (the copies in too, unless the caller declared its input ready; slot
  // reuse across calls is ordered by the per-slot events either way).
  cudaError_t e = cudaSuccess;
  if ((plan->flags & RR_HOST_CHAIN_INPUT_READY) == 0) {
    e = cudaEventRecord(plan->entry, s);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(plan->h2d, plan->entry, 0);
    if (e != cudaSuccess) return st(RR_CUDA_ERROR, "host chain ordering failed", e);
  }
  const int chunks = tokens == 0 ? 0 : (tokens + plan->chunk - 1) / plan->chunk;
  for (int c = 0; c < chunks; ++c) {
    const int i = c & 1;
    const rr_host_chain::Slot& sl = plan->slot[i];
    const long long t0 = static_cast<long long>(c) * plan->chunk;
    const int n = static_cast<int>(tokens - t0 < plan->chunk ? tokens - t0 : plan->chunk);
    // Host -> device: X of this chunk once the chain two chunks back is done.
    e = cudaStreamWaitEvent(plan->h2d, plan->compute_done[i], 0);
    if (e == cudaSuccess) {
      e = cudaMemcpyAsync(sl.x, x_host + t0 * K, sizeof(float) * n * K, cudaMemcpyHostToDevice,
                          plan->h2d);
    }
    if (e == cudaSuccess) e = cudaEventRecord(plan->h2d_done[i], plan->h2d);
    // The chain, once X has landed and the slot's previous Y has been read.
    if (e == cudaSuccess) e = cudaStreamWaitEvent(s, plan->h2d_done[i], 0);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(s, plan->d2h_done[i], 0);
    if (e != cudaSuccess) return st(RR_CUDA_ERROR, "host chain copy-in failed", e);
    rr_context cc = *ctx;
    cc.workspace = sl.workspace;
    cc.workspace_bytes = plan->workspace_bytes;
    const rr_status r = rr_chain_from_tokens(sl.x, router_weights, logit_bias, expert_weights,
                                             sl.logits, sl.ids, sl.weights, sl.counts,
                                             sl.offsets, sl.x_permuted, sl.route_pos,
                                             sl.y_permuted, sl.y, n, K, E, N, &cc);
    if (r.code != RR_SUCCESS) return r;
    e = cudaEventRecord(plan->compute_done[i], s);
    // Device -> host: Y (and the routing decisions when asked for).
    if (e == cudaSuccess) e = cudaStreamWaitEvent(plan->d2h, plan->compute_done[i], 0);
    if (e == cudaSuccess) {
      e = cudaMemcpyAsync(y_host + t0 * N, sl.y, sizeof(float) * n * N, cudaMemcpyDeviceToHost,
                          plan->d2h);
    }
    if (e == cudaSuccess && expert_ids_host != nullptr) {
      e = cudaMemcpyAsync(expert_ids_host + 2 * t0, sl.ids, sizeof(int32_t) * 2 * n,
                          cudaMemcpyDeviceToHost, plan->d2h);
    }
    if (e == cudaSuccess && route_weights_host != nullptr) {
      e = cudaMemcpyAsync(route_weights_host + 2 * t0, sl.weights, sizeof(float) * 2 * n,
                          cudaMemcpyDeviceToHost, plan->d2h);
    }
    if (e == cudaSuccess) e = cudaEventRecord(plan->d2h_done[i], plan->d2h);
    if (e != cudaSuccess) return st(RR_CUDA_ERROR, "host chain copy-out failed", e);
  }
  // Completion is ordered on ctx->stream.
  for (int i = 0; i < 2 && e == cudaSuccess; ++i) e = cudaStreamWaitEvent(s, plan->d2h_done[i], 0);
  if (e != cudaSuccess) return st(RR_CUDA_ERROR, "host chain completion ordering failed", e);
  return st(RR_SUCCESS, "success");
}

}  // extern "C"
