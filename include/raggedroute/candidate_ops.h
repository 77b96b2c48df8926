#pragma once

// Candidate (research) launchers that the reference's benchmark adapters and
// L3 chain call directly, outside the public operator API. Every one runs the
// B200 kernel of its operator; implementation ids select nothing but are
// validated as the reference does, so an adapter that passes an id the
// reference rejects still gets cudaErrorInvalidValue. Declarations equal the
// reference's internal headers so that its adapters link unchanged.
//
// Differences, all deliberate: experts up to 1024 (the reference stops at 64);
// token_permute places routes in the stable (route-ascending) order, which is
// one of the orders the reference's set-based checks accept, and uses the
// caller's pre-zeroed cursors (E int32) as its only scratch, leaving them
// equal to the per-expert counts.

#include <cuda_runtime_api.h>

#include <cstdint>

namespace raggedroute::ops {

// src/topk_gate/cuda_candidate/optimized_internal.h:19-21; ids 1..4.
cudaError_t launch_topk_gate_optimized(const float* logits, std::int32_t* expert_ids,
                                       float* weights, int tokens, int experts,
                                       std::uint32_t implementation_id, cudaStream_t caller_stream);

// src/histogram/cuda_candidate/optimized_internal.h:46-48; ids 101..104.
// Always overwrites counts, which satisfies both of the reference's output
// contracts for these ids (overwrite, or accumulate into caller-zeroed counts).
cudaError_t launch_histogram_optimized(const std::int32_t* expert_ids, std::int32_t* counts,
                                       int route_pairs, int experts,
                                       std::uint32_t implementation_id, cudaStream_t caller_stream);

// src/permute/cuda_candidate/optimized_internal.h:61-65; ids 1..10.
cudaError_t launch_token_permute_optimized(
    const float* x, const std::int32_t* expert_ids, const std::int32_t* offsets,
    std::int32_t* cursors, float* x_permuted, std::int32_t* route_pos,
    std::int32_t* sorted_route, int tokens, int experts, int top_k, int hidden,
    std::uint32_t implementation_id, cudaStream_t caller_stream);

// src/grouped_gemm/cuda_candidate/grouped_optimized_internal.h:31-34; ids 1..8.
cudaError_t launch_grouped_gemm_optimized(
    const float* x_permuted, const float* expert_weights, const std::int32_t* offsets,
    float* y_permuted, int experts, int hidden, int output, int max_expert_tokens,
    std::uint32_t implementation_id, cudaStream_t caller_stream);

// src/grouped_gemm/cuda_candidate/grouped_optimized_internal.h:91-94.
cudaError_t launch_grouped_gemm_sm86_fp32_v10_wave_aware_portfolio(
    const float* x_permuted, const float* expert_weights, const std::int32_t* offsets,
    float* y_permuted, int experts, int hidden, int output, int max_expert_tokens,
    int route_pairs, cudaStream_t caller_stream);

// src/unpermute/cuda_candidate/optimized_internal.h:11-15.
cudaError_t launch_unpermute_optimized(const float* y_permuted, const std::int32_t* route_pos,
                                       const float* route_weights, float* y, int tokens,
                                       int top_k, int output, cudaStream_t caller_stream);

// src/dense_gemm/cuda_candidate/optimized_internal.h:30-32; ids 1..7.
cudaError_t launch_dense_gemm_optimized(const float* a, const float* b, float* c, int m, int n,
                                        int k, std::uint32_t implementation_id,
                                        cudaStream_t caller_stream);

}  // namespace raggedroute::ops
