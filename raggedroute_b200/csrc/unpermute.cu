// Weighted unpermute (combine) for B200.
//
// y[t, c] = sum_{k < top_k} w[t*top_k + k] * y_permuted[route_pos[t*top_k + k], c],
// accumulated in rank order k = 0, 1, ... from 0.0f
// (src/unpermute/cuda_naive/baseline.cu:13-30; the CPU reference
// src/unpermute/cpu_reference/reference.cpp:10-37 sums the same terms in
// double). Each term is the rounded product w * v, added with
// round-to-nearest and subnormal operands and results flushed to zero: the
// arithmetic of the global float reduction that the grouped GEMM's fused
// combine uses, so the fused and the separate chains agree bit for bit
// (products and sums below 2^-126 in magnitude become zero; the reference's
// fused multiply-add keeps them). No atomics: each output row is produced by
// one warp, so results are bitwise reproducible.
//
// Design: one warp per token; the token's route positions and weights are
// fetched once per warp and broadcast by shuffle; each lane owns 128-bit
// column groups, so every gathered y_permuted row is read with coalesced
// 512-byte warp transactions and y is written once. HBM-bound: 4*R*N bytes
// gathered + 8*R bytes of metadata + 4*T*N bytes written.
#include "common.cuh"

namespace rrb {
namespace {

constexpr int kThreads = 256;

template <bool kVec, int kMaxK>
__global__ void __launch_bounds__(kThreads) unpermute_kernel(const float* __restrict__ yp,
                                                             const int32_t* __restrict__ route_pos,
                                                             const float* __restrict__ rw,
                                                             float* __restrict__ y, int tokens,
                                                             int top_k, int output,
                                                             long long routes) {
  const int lane = threadIdx.x & 31;
  const long long warp = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const long long nwarps = (static_cast<long long>(gridDim.x) * blockDim.x) >> 5;
  for (long long t = warp; t < tokens; t += nwarps) {
    // Lane k holds route k's position and weight (top_k <= 32 here).
    int my_pos = -1;
    float my_w = 0.0f;
    if (lane < top_k) {
      my_pos = __ldg(route_pos + t * top_k + lane);
      my_w = __ldg(rw + t * top_k + lane);
      if (my_pos < 0 || my_pos >= routes) my_pos = -1;
    }
    long long pos[kMaxK];
    float w[kMaxK];
#pragma unroll
    for (int k = 0; k < kMaxK; ++k) {
      const int p = __shfl_sync(0xffffffffu, my_pos, k);
      pos[k] = p;
      w[k] = __shfl_sync(0xffffffffu, my_w, k);
    }
    float* out = y + t * output;
    if constexpr (kVec) {
      const int n4 = output >> 2;
      for (int i = lane; i < n4; i += 32) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int k = 0; k < kMaxK; ++k) {
          if (k < top_k && pos[k] >= 0) {
            const float4 v = __ldg(reinterpret_cast<const float4*>(yp + pos[k] * output) + i);
            acc.x = add_ftz(acc.x, __fmul_rn(w[k], v.x));
            acc.y = add_ftz(acc.y, __fmul_rn(w[k], v.y));
            acc.z = add_ftz(acc.z, __fmul_rn(w[k], v.z));
            acc.w = add_ftz(acc.w, __fmul_rn(w[k], v.w));
          }
        }
        reinterpret_cast<float4*>(out)[i] = acc;
      }
    } else {
      for (int c = lane; c < output; c += 32) {
        float acc = 0.0f;
#pragma unroll
        for (int k = 0; k < kMaxK; ++k) {
          if (k < top_k && pos[k] >= 0) {
            acc = add_ftz(acc, __fmul_rn(w[k], __ldg(yp + pos[k] * output + c)));
          }
        }
        out[c] = acc;
      }
    }
  }
}

// Generic top_k (up to 64): positions and weights re-read per column group.
__global__ void __launch_bounds__(kThreads) unpermute_wide_kernel(
    const float* __restrict__ yp, const int32_t* __restrict__ route_pos,
    const float* __restrict__ rw, float* __restrict__ y, int tokens, int top_k, int output,
    long long routes) {
  const int lane = threadIdx.x & 31;
  const long long warp = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const long long nwarps = (static_cast<long long>(gridDim.x) * blockDim.x) >> 5;
  for (long long t = warp; t < tokens; t += nwarps) {
    for (int c = lane; c < output; c += 32) {
      float acc = 0.0f;
      for (int k = 0; k < top_k; ++k) {
        const long long r = t * top_k + k;
        const int p = __ldg(route_pos + r);
        if (p >= 0 && p < routes) {
          acc = add_ftz(acc, __fmul_rn(__ldg(rw + r),
                                       __ldg(yp + static_cast<long long>(p) * output + c)));
        }
      }
      y[t * output + c] = acc;
    }
  }
}

template <bool kVec>
cudaError_t launch_k(const float* yp, const int32_t* route_pos, const float* rw, float* y,
                     int tokens, int top_k, int output, cudaStream_t stream, int blocks) {
  const long long routes = static_cast<long long>(tokens) * top_k;
  if (top_k <= 2) {
    unpermute_kernel<kVec, 2><<<blocks, kThreads, 0, stream>>>(yp, route_pos, rw, y, tokens,
                                                               top_k, output, routes);
  } else if (top_k <= 4) {
    unpermute_kernel<kVec, 4><<<blocks, kThreads, 0, stream>>>(yp, route_pos, rw, y, tokens,
                                                               top_k, output, routes);
  } else if (top_k <= 8) {
    unpermute_kernel<kVec, 8><<<blocks, kThreads, 0, stream>>>(yp, route_pos, rw, y, tokens,
                                                               top_k, output, routes);
  } else {
    unpermute_wide_kernel<<<blocks, kThreads, 0, stream>>>(yp, route_pos, rw, y, tokens, top_k,
                                                           output, routes);
  }
  note_launch();
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_unpermute(const float* y_permuted, const int32_t* route_pos,
                             const float* route_weights, float* y, int tokens, int top_k,
                             int output, cudaStream_t stream) {
  if (tokens <= 0 || output <= 0) return cudaSuccess;
  const int warps_per_block = kThreads / 32;
  int blocks = ceil_div(tokens, warps_per_block);
  const int cap = 16 * sm_count();
  if (blocks > cap) blocks = cap;
  const bool vec = output % 4 == 0 && aligned_to(y_permuted, 16) && aligned_to(y, 16);
  return vec ? launch_k<true>(y_permuted, route_pos, route_weights, y, tokens, top_k, output,
                              stream, blocks)
             : launch_k<false>(y_permuted, route_pos, route_weights, y, tokens, top_k, output,
                               stream, blocks);
}

}  // namespace rrb
