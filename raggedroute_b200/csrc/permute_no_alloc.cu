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
//   * size: kNoAllocScratchBytes (4 KB: the per-expert cursors of the
//     largest expert count, which is all the permute needs for any number
//     of tokens) per GPU, held by every GPU that loads the library until the
//     process exits;
//   * a call whose scratch need (rr_token_permute_workspace_size) exceeds it
//     fails with RR_INVALID_ARGUMENT before any launch; this size check
//     comes right after the shape checks, the rest of the validation is
//     rr_token_permute's own (dispatch checks first, so an empty call on an
//     unsupported device or with an unknown kernel variant is rejected);
//   * no cudaMalloc, cudaFree or allocating library routine is called;
//   * the kernels overwrite every scratch word they later read, so nothing
//     has to start at zero and no reset launch is needed;
//   * all calls share the one array per GPU, so calls that overlap on the
//     GPU (for example on two streams at once) race on it and must be
//     serialised by the caller;
//   * the array's device address belongs to a CUDA context: it is looked up
//     (cudaGetSymbolAddress, with the device current) on the first call in
//     each context -- the first call on a device, and again after that
//     device's context was reset (cudaDeviceReset) or replaced -- and cached
//     under the context's unique id, read from the call's stream. That first
//     call in a context should come before any stream capture.
#include <cuda.h>
#include <cuda_runtime.h>

#include <climits>
#include <cstdint>
#include <limits>
#include <mutex>
#include <utility>
#include <vector>

#include "../../include/raggedroute/dispatch.h"
#include "../../include/raggedroute_b200.h"
#include "common.cuh"

namespace rrb {
namespace {

constexpr std::size_t kNoAllocScratchBytes = kMaxExperts * sizeof(int32_t);

// The scratch itself. In host code `g_no_alloc_scratch` names a host-side
// stand-in, not device memory: only the address from cudaGetSymbolAddress
// may be handed to a kernel.
__device__ __align__(256) unsigned char g_no_alloc_scratch[kNoAllocScratchBytes];

// Driver queries used to identify the context a call launches into. They
// are fetched through the runtime's entry-point lookup, so the library
// still links no driver library.
using StreamGetCtxFn = CUresult (*)(CUstream, CUcontext*);
using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

struct DriverQueries {
  StreamGetCtxFn stream_get_ctx = nullptr;
  CtxGetCurrentFn ctx_get_current = nullptr;
  CtxGetIdFn ctx_get_id = nullptr;
  cudaError_t error = cudaSuccess;
};

template <typename Fn>
cudaError_t entry_point(const char* name, Fn* out) {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult found = cudaDriverEntryPointSymbolNotFound;
  const cudaError_t err = cudaGetDriverEntryPointByVersion(name, &fn, 12000, cudaEnableDefault,
                                                           &found);
  if (err != cudaSuccess) return err;
  if (found != cudaDriverEntryPointSuccess || fn == nullptr) return cudaErrorNotSupported;
  *out = reinterpret_cast<Fn>(fn);
  return cudaSuccess;
}

const DriverQueries& driver_queries() {
  static const DriverQueries q = [] {
    DriverQueries d;
    d.error = entry_point("cuStreamGetCtx", &d.stream_get_ctx);
    if (d.error == cudaSuccess) d.error = entry_point("cuCtxGetCurrent", &d.ctx_get_current);
    if (d.error == cudaSuccess) d.error = entry_point("cuCtxGetId", &d.ctx_get_id);
    if (d.error != cudaSuccess) cudaGetLastError();
    return d;
  }();
  return q;
}

// (context id, scratch address) pairs. Context ids are never reused within
// a process, so an entry of a destroyed context can never match again; the
// list is bounded and drops its oldest entry when full.
constexpr std::size_t kMaxCachedContexts = 64;
std::mutex g_cache_mutex;
std::vector<std::pair<unsigned long long, void*>> g_cache;

bool context_id(CUcontext ctx, unsigned long long* id) {
  return ctx != nullptr && driver_queries().ctx_get_id(ctx, id) == CUDA_SUCCESS;
}

bool stream_context_id(cudaStream_t stream, unsigned long long* id) {
  CUcontext ctx = nullptr;
  if (driver_queries().stream_get_ctx(reinterpret_cast<CUstream>(stream), &ctx) != CUDA_SUCCESS) {
    return false;
  }
  return context_id(ctx, id);
}

// The scratch array's address in the context that `stream` belongs to.
cudaError_t scratch_for_stream(cudaStream_t stream, void** out) {
  const DriverQueries& d = driver_queries();
  if (d.error != cudaSuccess) return d.error;
  unsigned long long id = 0;
  if (stream_context_id(stream, &id)) {
    std::lock_guard<std::mutex> lock(g_cache_mutex);
    for (const auto& entry : g_cache) {
      if (entry.first == id) {
        *out = entry.second;
        return cudaSuccess;
      }
    }
  }
  // First call in this context: the lookup makes the current device's
  // context current on this thread (creating it if needed) and loads the
  // module there; the stream must belong to that same context.
  void* p = nullptr;
  cudaError_t err = cudaGetSymbolAddress(&p, g_no_alloc_scratch);
  if (err != cudaSuccess) {
    cudaGetLastError();
    return err;
  }
  CUcontext current = nullptr;
  unsigned long long current_id = 0;
  if (d.ctx_get_current(&current) != CUDA_SUCCESS || !context_id(current, &current_id) ||
      !stream_context_id(stream, &id)) {
    return cudaErrorDeviceUninitialized;
  }
  if (id != current_id) return cudaErrorInvalidResourceHandle;
  std::lock_guard<std::mutex> lock(g_cache_mutex);
  if (g_cache.size() >= kMaxCachedContexts) g_cache.erase(g_cache.begin());
  g_cache.emplace_back(id, p);
  *out = p;
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
  // Shape checks of rr_token_permute, so that the size query below is
  // defined; rr_token_permute repeats them.
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
                "token_permute_no_alloc: scratch need exceeds the 4 KB static array; "
                "use rr_token_permute with a caller workspace");
  }
  // The dispatch checks of rr_token_permute (architecture, kernel family
  // and research id) come before the empty-call return, as they do there.
  raggedroute::DeviceArchitecture arch = raggedroute::DeviceArchitecture::kOther;
  raggedroute::Status status = raggedroute::resolve_device_architecture(
      static_cast<raggedroute::DeviceArchitecture>(ctx->architecture), &arch);
  if (status.ok()) {
    raggedroute::DispatchRequest request;
    request.operator_kind = raggedroute::OperatorKind::kTokenPermute;
    request.architecture = arch;
    request.requested_kernel.family = static_cast<raggedroute::KernelFamily>(ctx->kernel_family);
    request.requested_kernel.implementation_id = ctx->implementation_id;
    request.signature.input = raggedroute::TensorSpec{};
    request.signature.output = raggedroute::TensorSpec{};
    raggedroute::DispatchDecision decision;
    status = raggedroute::select_kernel(request, &decision);
  }
  if (!status.ok()) {
    return make(static_cast<int32_t>(status.code), status.message, status.cuda_error);
  }
  if (tokens == 0) return make(RR_SUCCESS, "success");
  void* scratch = nullptr;
  const cudaError_t err = rrb::scratch_for_stream(static_cast<cudaStream_t>(ctx->stream),
                                                  &scratch);
  if (err != cudaSuccess) {
    return make(RR_CUDA_ERROR, "token_permute_no_alloc: scratch address lookup failed", err);
  }
  // The permute itself, with rr_token_permute's remaining checks (null
  // pointers, alignment, workspace size), on the static array.
  rr_context with_scratch = *ctx;
  with_scratch.workspace = scratch;
  with_scratch.workspace_bytes = rrb::kNoAllocScratchBytes;
  return rr_token_permute(x, expert_ids, offsets, x_permuted, route_pos, sorted_route, tokens,
                          experts, top_k, hidden, &with_scratch);
}

}  // extern "C"
