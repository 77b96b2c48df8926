// FP32 SIMT grouped GEMM: the exact-FP32 engine for shapes the tcgen05 path
// cannot take (row strides that are not a multiple of 16 bytes, misaligned
// buffers) and for tiny problems. Same contract as the reference
// (src/grouped_gemm/cuda_naive/baseline.cu:11-31): y[r, :] = x[r, :] . W[e]
// for r in [offsets[e], offsets[e+1]), FP32 FMA accumulation in k order, K = 0
// writes zeros, rows outside every segment are untouched.
//
// Persistent CTAs walk the device-side tile schedule (tile_sched.cuh). A CTA
// computes a 64x64 tile with 256 threads (4x4 outputs each) from 64x16 and
// 16x64 shared-memory stages.
#include "tile_sched.cuh"

namespace rrb {
namespace {

constexpr int kBM = 64;
constexpr int kBN = 64;
constexpr int kBK = 16;
constexpr int kThreads = 256;

__global__ void __launch_bounds__(kThreads) grouped_gemm_simt_kernel(
    const float* __restrict__ x, const float* __restrict__ w, const int32_t* __restrict__ offsets,
    float* __restrict__ y, int experts, int rows, int hidden, int output, int wsets,
    const RowScatter scatter, const RowGather gather) {
  __shared__ int prefix[kMaxExperts + 1];
  __shared__ int scratch[33];
  __shared__ float as[kBK][kBM + 4];
  __shared__ float bs[kBK][kBN + 4];
  const int n_tiles_n = (output + kBN - 1) / kBN;
  const int total = build_tile_prefix(offsets, experts, rows, kBM, n_tiles_n, prefix, scratch);
  const int tx = threadIdx.x % 16;  // column group
  const int ty = threadIdx.x / 16;  // row group
  for (int t = blockIdx.x; t < total; t += gridDim.x) {
    const TileCoord tc = tile_coord(t, offsets, experts, rows, prefix, kBM, kBN, n_tiles_n);
    const float* we = w + static_cast<long long>(tc.expert % wsets) * hidden * output;
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
    for (int k0 = 0; k0 < hidden; k0 += kBK) {
      // A stage: 64 rows x 16 k, transposed into as[k][m].
      for (int i = threadIdx.x; i < kBM * kBK; i += kThreads) {
        const int m = i / kBK;
        const int kk = i % kBK;
        const int r = tc.row0 + m;
        const int k = k0 + kk;
        long long src_row = r;
        if (gather.route != nullptr && r < tc.row_end) src_row = __ldg(gather.route + r) / gather.div;
        as[kk][m] = (r < tc.row_end && k < hidden) ? __ldg(x + src_row * hidden + k) : 0.0f;
      }
      // B stage: 16 k x 64 columns.
      for (int i = threadIdx.x; i < kBK * kBN; i += kThreads) {
        const int kk = i / kBN;
        const int n = i % kBN;
        const int k = k0 + kk;
        const int c = tc.col0 + n;
        bs[kk][n] = (k < hidden && c < output) ? __ldg(we + static_cast<long long>(k) * output + c)
                                               : 0.0f;
      }
      __syncthreads();
#pragma unroll
      for (int kk = 0; kk < kBK; ++kk) {
        float a[4], b[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) a[i] = as[kk][ty * 4 + i];
#pragma unroll
        for (int j = 0; j < 4; ++j) b[j] = bs[kk][tx * 4 + j];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
      }
      __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = tc.row0 + ty * 4 + i;
      if (r >= tc.row_end) continue;
      float* out = y + static_cast<long long>(r) * output;
      if (scatter.dst != nullptr) {
        if (scatter.abort != nullptr && *scatter.abort != 0) continue;
        out = scatter_row(scatter, r, output);
        if (out == nullptr) continue;
      }
      if (scatter.combine != nullptr) {
        float wgt;
        out = combine_row(scatter, r, output, wgt);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int c = tc.col0 + tx * 4 + j;
          if (c < output) red_add_f32(out + c, __fmul_rn(wgt, acc[i][j]));
        }
        continue;
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int c = tc.col0 + tx * 4 + j;
        if (c < output) out[c] = acc[i][j];
      }
    }
  }
  if (scatter.dst != nullptr) __threadfence_system();
}

}  // namespace

cudaError_t launch_grouped_gemm_simt(const float* x, const float* w, const int32_t* offsets,
                                     float* y, int experts, int rows, int hidden, int output,
                                     cudaStream_t stream, int weight_sets,
                                     const RowScatter* scatter, const RowGather* gather) {
  const int wsets = weight_sets > 0 ? weight_sets : experts;
  if (output <= 0) return cudaSuccess;
  int grid = 4 * sm_count();
  if (offsets == nullptr) {
    const long long tiles = static_cast<long long>((rows + kBM - 1) / kBM) *
                            ((output + kBN - 1) / kBN);
    if (tiles <= 0) return cudaSuccess;
    if (tiles < grid) grid = static_cast<int>(tiles);
  }
  grouped_gemm_simt_kernel<<<grid, kThreads, 0, stream>>>(x, w, offsets, y, experts, rows, hidden,
                                                          output, wsets,
                                                          scatter != nullptr ? *scatter
                                                                             : RowScatter{},
                                                          gather != nullptr ? *gather
                                                                            : RowGather{});
  note_launch();
  return cudaGetLastError();
}

}  // namespace rrb
