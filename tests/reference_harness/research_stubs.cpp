// TEST INFRASTRUCTURE of the reference-harness build (not part of the
// library). The reference's benchmark core (benchmarks/core/registry.cpp)
// links every research adapter, and those call research-only launchers of the
// reference's SM86 study: low-precision and mma.sync tensor-core GEMMs, the
// v4-v9 descriptor/balanced grouped GEMMs, fused permute preparations and
// copies, and a vLLM top-2 baseline. libraggedroute_b200 implements the
// operators, their public API, the naive launchers and the candidate
// launchers the L3 chain uses (include/raggedroute/candidate_ops.h), but not
// these research variants. Each stub below records its name and returns
// cudaErrorNotSupported, so the harness driver reports the variant that
// reached it as unsupported instead of failing or running another kernel.
// Declarations come from the reference's own headers (include path at build
// time), so the signatures are the reference's.
#include <cuda_runtime_api.h>

#include <cstddef>
#include <cstdint>

#include "common/tensorcore_gemm.h"
#include "grouped_gemm/cuda_candidate/grouped_optimized_internal.h"
#include "permute/cuda_candidate/optimized_internal.h"
#include "raggedroute/benchmark/library_baselines.h"

namespace harness {
// Name of the last research stub that was reached (nullptr: none).
const char* g_last_research_stub = nullptr;
}  // namespace harness

#define RR_HARNESS_STUB(name)             \
  do {                                    \
    harness::g_last_research_stub = name; \
    return cudaErrorNotSupported;         \
  } while (0)

namespace raggedroute::ops {

cudaError_t launch_dense_gemm_tensorcore(const void*, const void*, float*, int, int, int,
                                         ScalarType, const TensorCoreConfig&, cudaStream_t) {
  RR_HARNESS_STUB("launch_dense_gemm_tensorcore");
}
cudaError_t launch_grouped_gemm_tensorcore(const void*, const void*, const std::int32_t*, float*,
                                           int, int, int, int, ScalarType,
                                           const TensorCoreConfig&, cudaStream_t) {
  RR_HARNESS_STUB("launch_grouped_gemm_tensorcore");
}
cudaError_t launch_dense_gemm_lowp_simt(const void*, const void*, float*, int, int, int,
                                        ScalarType, cudaStream_t) {
  RR_HARNESS_STUB("launch_dense_gemm_lowp_simt");
}
cudaError_t launch_grouped_gemm_lowp_simt(const void*, const void*, const std::int32_t*, float*,
                                          int, int, int, int, ScalarType, cudaStream_t) {
  RR_HARNESS_STUB("launch_grouped_gemm_lowp_simt");
}
cudaError_t launch_gemm_quantize(const float*, void*, std::size_t, ScalarType, cudaStream_t) {
  RR_HARNESS_STUB("launch_gemm_quantize");
}

#define RR_HARNESS_BALANCED(fn)                                                               \
  cudaError_t fn(const float*, const float*, const std::int32_t*, float*, int, int, int, int, \
                 int, cudaStream_t) {                                                         \
    RR_HARNESS_STUB(#fn);                                                                     \
  }
RR_HARNESS_BALANCED(launch_grouped_gemm_sm86_fp32_v5_balanced_direct)
RR_HARNESS_BALANCED(launch_grouped_gemm_sm86_fp32_v6_balanced_32x128)
RR_HARNESS_BALANCED(launch_grouped_gemm_sm86_fp32_v8_balanced_16x128)
RR_HARNESS_BALANCED(launch_grouped_gemm_sm86_fp32_v9_balanced_32x64)

std::size_t grouped_gemm_descriptor_workspace_size(int, int, int) noexcept {
  harness::g_last_research_stub = "grouped_gemm_descriptor_workspace_size";
  return 0;
}
cudaError_t launch_grouped_gemm_sm86_fp32_v4_descriptor(const float*, const float*,
                                                        const std::int32_t*, float*, int, int,
                                                        int, int, void*, std::size_t,
                                                        std::uint32_t, cudaStream_t) {
  RR_HARNESS_STUB("launch_grouped_gemm_sm86_fp32_v4_descriptor");
}

cudaError_t launch_token_permute_prepare_offsets_fused(const std::int32_t*, std::int32_t*,
                                                       std::int32_t*, std::int32_t*, int, int,
                                                       int, cudaStream_t) {
  RR_HARNESS_STUB("launch_token_permute_prepare_offsets_fused");
}
cudaError_t launch_token_permute_routeprep_shared_rank(const std::int32_t*, std::int32_t*,
                                                       std::int32_t*, std::int32_t*,
                                                       std::int32_t*, int, int, int, int,
                                                       cudaStream_t) {
  RR_HARNESS_STUB("launch_token_permute_routeprep_shared_rank");
}
cudaError_t launch_token_permute_copy_token_owned_topk(const float*, const std::int32_t*, float*,
                                                       int, int, int, cudaStream_t) {
  RR_HARNESS_STUB("launch_token_permute_copy_token_owned_topk");
}
cudaError_t launch_token_permute_copy_from_positions(const float*, const std::int32_t*, float*,
                                                     int, int, int, cudaStream_t) {
  RR_HARNESS_STUB("launch_token_permute_copy_from_positions");
}

}  // namespace raggedroute::ops

namespace raggedroute::benchmark::library_baseline {

bool supports_vllm_row_packed_top2(int, const float*) noexcept {
  harness::g_last_research_stub = "supports_vllm_row_packed_top2";
  return false;
}
cudaError_t launch_vllm_row_packed_top2(const float*, std::int32_t*, float*, int, int,
                                        cudaStream_t) {
  RR_HARNESS_STUB("launch_vllm_row_packed_top2");
}

}  // namespace raggedroute::benchmark::library_baseline
