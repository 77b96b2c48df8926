// Grouped GEMM engine selection. The tcgen05 3xTF32 engine is added next;
// until then every shape takes the exact-FP32 SIMT engine.
#include "common.cuh"

namespace rrb {

bool tc_gemm_supported(const float*, const float*, const float*, int, int) { return false; }

cudaError_t launch_grouped_gemm_tc(const float*, const float*, const int32_t*, float*, int, int,
                                   int, int, cudaStream_t) {
  return cudaErrorNotSupported;
}

cudaError_t launch_grouped_gemm(const float* x, const float* w, const int32_t* offsets, float* y,
                                int experts, int rows, int hidden, int output,
                                cudaStream_t stream) {
  if (tc_gemm_supported(x, w, y, hidden, output)) {
    return launch_grouped_gemm_tc(x, w, offsets, y, experts, rows, hidden, output, stream);
  }
  return launch_grouped_gemm_simt(x, w, offsets, y, experts, rows, hidden, output, stream);
}

}  // namespace rrb
