// Shared device helpers and the internal launcher interface of
// libraggedroute_b200. Every launcher here enqueues on the given stream,
// performs no allocation and no host synchronization, and returns the launch
// status from cudaGetLastError().
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace rrb {

constexpr int kMaxExperts = 1024;
constexpr int kNumSms = 148;  // B200; the launchers query the real count once.

// Bits of the device error word (set by bounded waits, read by
// rr_consume_device_error).
constexpr unsigned kErrMbarTimeout = 1u << 0;
constexpr unsigned kErrTmemAlloc = 1u << 1;
constexpr unsigned kErrScheduler = 1u << 2;

// Counts every kernel this library launches (for the bench's launch claim).
void note_launch(int n = 1);
int sm_count();
unsigned* device_error_word();

__device__ __forceinline__ void raise_device_error(unsigned* word, unsigned bits) {
  if (word != nullptr) atomicOr(word, bits);
}

__device__ __forceinline__ unsigned lanemask_lt() {
  unsigned m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

inline bool aligned_to(const void* p, std::size_t a) {
  return (reinterpret_cast<std::uintptr_t>(p) % a) == 0;
}

inline int ceil_div(long long a, long long b) { return static_cast<int>((a + b - 1) / b); }

// ---- launchers (implemented in the .cu files) -------------------------------

// topk_gate.cu. remap (optional, [experts]) replaces each selected id by
// remap[id] on output (the expert-parallel runtime's virtual expert ids).
cudaError_t launch_topk_gate(const float* logits, const float* bias, int32_t* ids, float* weights,
                             int tokens, int experts, cudaStream_t stream,
                             const int32_t* remap = nullptr);

// routing.cu
cudaError_t launch_histogram_accumulate(const int32_t* ids, int32_t* counts, int routes,
                                        int experts, cudaStream_t stream);
cudaError_t launch_exclusive_scan(const int32_t* counts, int32_t* offsets, int experts,
                                  cudaStream_t stream);
// Fused histogram + exclusive scan; overwrites counts and offsets (reset is
// part of the call).
cudaError_t launch_histogram_exclusive_scan(const int32_t* ids, int32_t* counts,
                                            int32_t* offsets, int routes, int experts,
                                            cudaStream_t stream);

// Expert-parallel receive offsets (nranks * local <= 1024 groups).
cudaError_t launch_ep_recv_offsets(const int32_t* count_all, int32_t* recv_offsets, int nranks,
                                   int experts, int rank, int local, cudaStream_t stream);

// permute.cu
std::size_t permute_workspace_bytes(int tokens, int experts, int top_k);
// Stable permute; workspace holds >= permute_workspace_bytes(...) bytes and
// its first `experts` ints end as the per-expert counts.
cudaError_t launch_token_permute(const float* x, const int32_t* ids, const int32_t* offsets,
                                 float* x_permuted, int32_t* route_pos, int32_t* sorted_route,
                                 int tokens, int experts, int top_k, int hidden, void* workspace,
                                 cudaStream_t stream);
// Workspace-free stable permute for the low-level launcher: the expert count
// is unknown, cursors accumulate (caller zeroes them).
cudaError_t launch_token_permute_cursor(const float* x, const int32_t* ids,
                                        const int32_t* offsets, int32_t* cursors,
                                        float* x_permuted, int32_t* route_pos,
                                        int32_t* sorted_route, int tokens, int top_k, int hidden,
                                        cudaStream_t stream);

// unpermute.cu
cudaError_t launch_unpermute(const float* y_permuted, const int32_t* route_pos,
                             const float* route_weights, float* y, int tokens, int top_k,
                             int output, cudaStream_t stream);

// gemm_simt.cu / gemm_tc.cu
// Grouped GEMM with rows split by offsets[experts+1] (`experts` row groups);
// offsets == nullptr means one group covering `rows` rows (dense GEMM). Group
// g multiplies by weight set (g % weight_sets) of w[weight_sets, hidden,
// output]; weight_sets = 0 means one weight set per group. The
// expert-parallel runtime uses weight_sets < experts for its
// (source rank, local expert) groups.
cudaError_t launch_grouped_gemm(const float* x, const float* w, const int32_t* offsets,
                                float* y, int experts, int rows, int hidden, int output,
                                cudaStream_t stream, int weight_sets = 0);
cudaError_t launch_grouped_gemm_simt(const float* x, const float* w, const int32_t* offsets,
                                     float* y, int experts, int rows, int hidden, int output,
                                     cudaStream_t stream, int weight_sets = 0);
bool tc_gemm_supported(const float* x, const float* w, const float* y, int hidden, int output);
cudaError_t launch_grouped_gemm_tc(const float* x, const float* w, const int32_t* offsets,
                                   float* y, int experts, int rows, int hidden, int output,
                                   cudaStream_t stream, int weight_sets = 0);

// misc.cu
cudaError_t launch_cache_scrub(uint32_t* buffer, std::size_t elements, cudaStream_t stream);

}  // namespace rrb
