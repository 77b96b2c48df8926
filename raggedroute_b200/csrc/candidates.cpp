// The reference's candidate (research) launchers, raggedroute::ops::
// launch_*_optimized and the grouped-GEMM v10 portfolio, which its benchmark
// adapters and L3 chain call outside the public operator API
// (benchmarks/adapters/chain_adapter.cpp:417-463 and the operator adapters).
// Each validates its arguments and implementation id as the reference
// launcher does (cited per function) and then runs this library's B200
// kernel for the operator through the matching low-level launcher.
#include <cuda_runtime.h>

#include <cstdint>
#include <limits>

#include "../../include/raggedroute/baseline_ops.h"
#include "../../include/raggedroute/candidate_ops.h"
#include "common.cuh"

namespace raggedroute::ops {

// src/topk_gate/cuda_candidate/optimized.cu:454-478 (ids 1..4).
cudaError_t launch_topk_gate_optimized(const float* logits, std::int32_t* expert_ids,
                                       float* weights, int tokens, int experts,
                                       std::uint32_t implementation_id,
                                       cudaStream_t caller_stream) {
  if (tokens < 0 || experts < 2 || experts > rrb::kMaxExperts || implementation_id < 1 ||
      implementation_id > 4) {
    return cudaErrorInvalidValue;
  }
  return launch_topk_gate_naive(logits, expert_ids, weights, tokens, experts, caller_stream);
}

// src/histogram/cuda_candidate/optimized.cu:89-126 (ids 101..104). The
// reference's ids either overwrite counts or accumulate into counts the
// caller zeroed (histogram_optimized_requires_external_reset); overwriting
// gives the same counts in both cases.
cudaError_t launch_histogram_optimized(const std::int32_t* expert_ids, std::int32_t* counts,
                                       int route_pairs, int experts,
                                       std::uint32_t implementation_id,
                                       cudaStream_t caller_stream) {
  if (route_pairs < 0 || experts <= 0 || experts > rrb::kMaxExperts) {
    return cudaErrorInvalidValue;
  }
  if (route_pairs > 0 && (expert_ids == nullptr || counts == nullptr)) {
    return cudaErrorInvalidValue;
  }
  if (implementation_id < 101 || implementation_id > 104) return cudaErrorInvalidValue;
  if (counts == nullptr) return cudaErrorInvalidValue;
  return rrb::launch_histogram(expert_ids, counts, route_pairs, experts, caller_stream);
}

// src/permute/cuda_candidate/optimized.cu:419-437, 649-719 (ids 1..10).
// Cursors: caller-zeroed E int32, ending equal to the per-expert counts.
cudaError_t launch_token_permute_optimized(
    const float* x, const std::int32_t* expert_ids, const std::int32_t* offsets,
    std::int32_t* cursors, float* x_permuted, std::int32_t* route_pos,
    std::int32_t* sorted_route, int tokens, int experts, int top_k, int hidden,
    std::uint32_t implementation_id, cudaStream_t caller_stream) {
  if (tokens < 0 || experts <= 0 || experts > rrb::kMaxExperts || top_k <= 0 ||
      top_k > experts || hidden < 0 || implementation_id < 1 || implementation_id > 10) {
    return cudaErrorInvalidValue;
  }
  if (tokens == 0) return cudaSuccess;
  if (tokens > std::numeric_limits<int>::max() / top_k) return cudaErrorInvalidValue;
  if (expert_ids == nullptr || offsets == nullptr || cursors == nullptr || route_pos == nullptr ||
      (hidden != 0 && (x == nullptr || x_permuted == nullptr))) {
    return cudaErrorInvalidValue;
  }
  return launch_token_permute_naive(x, expert_ids, offsets, cursors, x_permuted, route_pos,
                                    sorted_route, tokens, top_k, hidden, caller_stream);
}

// src/grouped_gemm/cuda_candidate/optimized.cu:227-286 (ids 1..8).
cudaError_t launch_grouped_gemm_optimized(
    const float* x_permuted, const float* expert_weights, const std::int32_t* offsets,
    float* y_permuted, int experts, int hidden, int output, int max_expert_tokens,
    std::uint32_t implementation_id, cudaStream_t caller_stream) {
  if (implementation_id < 1 || implementation_id > 8) return cudaErrorInvalidValue;
  return launch_grouped_gemm_naive(x_permuted, expert_weights, offsets, y_permuted, experts,
                                   hidden, output, max_expert_tokens, caller_stream);
}

// src/grouped_gemm/cuda_candidate/optimized_balanced_wide.cu:363-396.
cudaError_t launch_grouped_gemm_sm86_fp32_v10_wave_aware_portfolio(
    const float* x_permuted, const float* expert_weights, const std::int32_t* offsets,
    float* y_permuted, int experts, int hidden, int output, int max_expert_tokens,
    int route_pairs, cudaStream_t caller_stream) {
  if (experts <= 0 || experts > rrb::kMaxExperts || hidden < 0 || output < 0 ||
      max_expert_tokens < 0) {
    return cudaErrorInvalidValue;
  }
  if (max_expert_tokens == 0 || output == 0) return cudaSuccess;
  if (route_pairs <= 0 || max_expert_tokens > route_pairs) return cudaErrorInvalidValue;
  return launch_grouped_gemm_naive(x_permuted, expert_weights, offsets, y_permuted, experts,
                                   hidden, output, max_expert_tokens, caller_stream);
}

// src/unpermute/cuda_candidate/optimized.cu:107-140.
cudaError_t launch_unpermute_optimized(const float* y_permuted, const std::int32_t* route_pos,
                                       const float* route_weights, float* y, int tokens,
                                       int top_k, int output, cudaStream_t caller_stream) {
  if (tokens < 0 || top_k <= 0 || top_k > 64 || output < 0) return cudaErrorInvalidValue;
  return launch_unpermute_naive(y_permuted, route_pos, route_weights, y, tokens, top_k, output,
                                caller_stream);
}

// src/dense_gemm/cuda_candidate/optimized.cu:235-270 (ids 1..7).
cudaError_t launch_dense_gemm_optimized(const float* a, const float* b, float* c, int m, int n,
                                        int k, std::uint32_t implementation_id,
                                        cudaStream_t caller_stream) {
  if (implementation_id < 1 || implementation_id > 7) return cudaErrorInvalidValue;
  return launch_dense_gemm_naive(a, b, c, m, n, k, caller_stream);
}

}  // namespace raggedroute::ops
