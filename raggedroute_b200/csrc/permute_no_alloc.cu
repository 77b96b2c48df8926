// token_permute for callers that cannot allocate device memory.
//
// Some callers of this library have no way to hand it a workspace: an
// inference engine whose memory planner owns every device byte and forbids
// allocations after start-up, or a host-language binding that can pass
// buffers it already has but cannot reach a CUDA allocator. For them,
// rr_token_permute_no_alloc runs the same stable permute as rr_token_permute
// with its scratch (the per-expert cursors and the per-chunk expert table)
// in a fixed array that lives in this library's device image:
//
//   * size: kNoAllocScratchBytes (4 MiB) per GPU, held by every GPU that
//     loads the library until the process exits;
//   * a call whose scratch need (rr_token_permute_workspace_size) exceeds it
//     fails with RR_INVALID_ARGUMENT before any launch;
//   * no cudaMalloc, cudaFree or allocating library routine is called;
//   * the kernels overwrite every scratch word they later read, so nothing
//     has to start at zero and no reset launch is needed;
//   * all calls share the one array per GPU, so calls that overlap on the
//     GPU (for example on two streams at once) race on it and must be
//     serialised by the caller;
//   * the array's device address is looked up on the first call on each
//     device, with that device current (cudaGetSymbolAddress). That first
//     call should come before any stream capture.
#include <cuda_runtime.h>

#include <climits>
#include <cstdint>
#include <limits>
#include <mutex>

#include "../../include/raggedroute_b200.h"
#include "common.cuh"

namespace rrb {
namespace {

constexpr std::size_t kNoAllocScratchBytes = 4u << 20;
constexpr int kMaxDevices = 64;

// The scratch itself. In host code `g_no_alloc_scratch` names a host-side
// stand-in, not device memory: only the address from cudaGetSymbolAddress
// may be handed to a kernel.
__device__ __align__(256) unsigned char g_no_alloc_scratch[kNoAllocScratchBytes];

std::once_flag g_once[kMaxDevices];
void* g_scratch_ptr[kMaxDevices] = {};
cudaError_t g_lookup_error[kMaxDevices] = {};

// Resolves the array's device address for the current device (once).
cudaError_t scratch_for_current_device(void** out) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return err;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::call_once(g_once[dev], [dev] {
    void* p = nullptr;
    g_lookup_error[dev] = cudaGetSymbolAddress(&p, g_no_alloc_scratch);
    if (g_lookup_error[dev] == cudaSuccess) {
      g_scratch_ptr[dev] = p;
    } else {
      cudaGetLastError();
    }
  });
  if (g_lookup_error[dev] != cudaSuccess) return g_lookup_error[dev];
  *out = g_scratch_ptr[dev];
  return cudaSuccess;
}

rr_status make(int32_t code, const char* msg, cudaError_t e = cudaSuccess) {
  rr_status s;
  s.code = code;
  s.cuda_error = static_cast<int32_t>(e);
  s.message = msg;
  return s;
}

}  // namespace
}  // namespace rrb

extern "C" {

// No reference counterpart (see include/raggedroute_b200.h).
rr_status rr_token_permute_no_alloc(const float* x, const int32_t* expert_ids,
                                    const int32_t* offsets, float* x_permuted, int32_t* route_pos,
                                    int32_t* sorted_route, int tokens, int experts, int top_k,
                                    int hidden, const rr_context* ctx) {
  using rrb::make;
  if (ctx == nullptr) return make(RR_INVALID_ARGUMENT, "rr_context must not be null");
  // Shape checks and their order follow rr_token_permute.
  if (tokens < 0 || experts <= 0 || experts > rrb::kMaxExperts || top_k <= 0 ||
      top_k > experts || hidden < 0) {
    return make(RR_INVALID_ARGUMENT,
                "token_permute requires T>=0, 1<=top_k<=E<=1024, and hidden>=0");
  }
  if (tokens > 0 && tokens > std::numeric_limits<int>::max() / top_k) {
    return make(RR_INVALID_ARGUMENT, "token_permute route count exceeds int32 indexing");
  }
  const std::size_t need = rrb::permute_workspace_bytes(tokens, experts, top_k);
  if (need > rrb::kNoAllocScratchBytes) {
    return make(RR_INVALID_ARGUMENT,
                "token_permute_no_alloc: scratch need exceeds the 4 MiB static array; "
                "use rr_token_permute with a caller workspace");
  }
  if (tokens == 0) return make(RR_SUCCESS, "success");
  if (expert_ids == nullptr || offsets == nullptr || route_pos == nullptr ||
      (hidden != 0 && (x == nullptr || x_permuted == nullptr))) {
    return make(RR_INVALID_ARGUMENT, "token_permute received a null device pointer");
  }
  if (!rrb::aligned_to(x, 4) || !rrb::aligned_to(x_permuted, 4)) {
    return make(RR_INVALID_ARGUMENT, "token_permute FP32 buffers must be 4-byte aligned");
  }
  int32_t arch = ctx->architecture;
  if (arch == RR_ARCH_AUTO) {
    const rr_status q = rr_query_current_device_architecture(&arch);
    if (q.code != RR_SUCCESS) return q;
  }
  if (arch != RR_ARCH_SM100) {
    return make(RR_UNSUPPORTED_ARCHITECTURE, "libraggedroute_b200 ships sm_100a kernels only");
  }
  void* scratch = nullptr;
  cudaError_t err = rrb::scratch_for_current_device(&scratch);
  if (err != cudaSuccess) {
    return make(RR_CUDA_ERROR, "token_permute_no_alloc: scratch address lookup failed", err);
  }
  err = rrb::launch_token_permute(x, expert_ids, offsets, x_permuted, route_pos, sorted_route,
                                  tokens, experts, top_k, hidden, scratch,
                                  static_cast<cudaStream_t>(ctx->stream));
  if (err != cudaSuccess) {
    return make(RR_CUDA_ERROR, "token_permute_no_alloc kernel launch failed", err);
  }
  return make(RR_SUCCESS, "success");
}

}  // extern "C"
