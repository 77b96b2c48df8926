// Prepared expert weights for the tcgen05 grouped GEMM (new: no reference
// counterpart).
//
// For weights that stay fixed across calls (inference), the 3xTF32 split of
// B can be done once: W [E][K][N] (N contiguous) is written as two K-major
// arrays [E][N][K], hi = W and lo = W - trunc(W), where trunc clears the low
// 13 mantissa bits (the value a kind::tf32 MMA reads from FP32 bits, so hi
// needs no rounding of its own). The grouped GEMM then TMA-loads both B
// operands in the layout its MMAs read and splits only the token rows.
// One pass, HBM-bound: E*K*N*4 bytes read, twice that written.
#include "common.cuh"

namespace rrb {
namespace {

constexpr int kTile = 32;

// 32 x 32 tiles of one expert through shared memory: loads along N, stores
// along K, both coalesced. Out-of-range elements are skipped.
__global__ void __launch_bounds__(256) prepare_weights_kernel(const float* __restrict__ w,
                                                              float* __restrict__ hi,
                                                              float* __restrict__ lo, int hidden,
                                                              int output) {
  __shared__ float tile[kTile][kTile + 1];
  const long long e = blockIdx.z;
  const int n0 = blockIdx.x * kTile;
  const int k0 = blockIdx.y * kTile;
  const float* src = w + e * hidden * static_cast<long long>(output);
  const long long dst_base = e * output * static_cast<long long>(hidden);
#pragma unroll
  for (int j = 0; j < kTile; j += 8) {
    const int k = k0 + threadIdx.y + j;
    const int n = n0 + threadIdx.x;
    if (k < hidden && n < output) {
      tile[threadIdx.y + j][threadIdx.x] = __ldg(src + static_cast<long long>(k) * output + n);
    }
  }
  __syncthreads();
#pragma unroll
  for (int j = 0; j < kTile; j += 8) {
    const int n = n0 + threadIdx.y + j;
    const int k = k0 + threadIdx.x;
    if (k < hidden && n < output) {
      const float v = tile[threadIdx.x][threadIdx.y + j];
      const float t = __uint_as_float(__float_as_uint(v) & 0xFFFFE000u);
      const long long o = dst_base + static_cast<long long>(n) * hidden + k;
      hi[o] = v;
      lo[o] = v - t;
    }
  }
}

}  // namespace

std::size_t prepared_weights_half_bytes(int experts, int hidden, int output) {
  const std::size_t b = static_cast<std::size_t>(experts) * static_cast<std::size_t>(hidden) *
                        static_cast<std::size_t>(output) * sizeof(float);
  return (b + 255) & ~static_cast<std::size_t>(255);
}

cudaError_t launch_prepare_weights(const float* w, float* hi, float* lo, int experts, int hidden,
                                   int output, cudaStream_t stream) {
  if (experts <= 0 || hidden <= 0 || output <= 0) return cudaSuccess;
  const dim3 grid(static_cast<unsigned>(ceil_div(output, kTile)),
                  static_cast<unsigned>(ceil_div(hidden, kTile)), static_cast<unsigned>(experts));
  prepare_weights_kernel<<<grid, dim3(kTile, 8), 0, stream>>>(w, hi, lo, hidden, output);
  note_launch();
  return cudaGetLastError();
}

}  // namespace rrb
