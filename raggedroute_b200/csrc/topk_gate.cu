// Top-2 selected-softmax gate for B200.
//
// Semantics (src/topk_gate/cuda_naive/baseline.cu:18-80 and
// src/topk_gate/cpu_reference/reference.cpp:12-72 of the reference): per row,
// NaN reads as -inf, the larger value wins, equal values go to the lower
// expert id; an all-NaN row gives ids {0,1} and weights {0.5,0.5}; equal
// selected values give {0.5,0.5}; first == +inf or second == -inf gives
// {1,0}; otherwise r = exp(second - first), w0 = 1/(1+r), w1 = r*w0.
//
// Design: a row is owned by a group of L lanes (L = 1..32, a power of two) so
// one warp covers 32/L rows and every lane issues 128-bit loads when the row
// stride allows it. A candidate is (value, expert id) with NaN read as -inf
// and -0 as +0; (v, e) precedes (w, f) when v > w, or v == w and e < f. A
// lane sees its candidates in increasing id order, so inside a lane a later
// candidate with an equal value never precedes an earlier one and one float
// compare decides; the L partial top-2 lists of a row merge by xor shuffles
// with the full rule. An all-NaN row therefore ranks ids 0 and 1 (both -inf,
// lower ids first) with equal values, which is the reference's {0,1} /
// {0.5,0.5} outcome. The grid is one resident wave; CTAs loop over row
// groups, so no second, partly filled wave of CTAs trails the first. The
// kernel is HBM-bound: 4*E bytes in and 16 bytes out per row. An optional
// remap table rewrites each selected id on output (the expert-parallel
// runtime's replicated "virtual" experts).
#include <limits>

#include "common.cuh"

namespace rrb {
namespace {

constexpr float kNegInf = -std::numeric_limits<float>::infinity();

__device__ __forceinline__ float canonical(float v) { return v != v ? kNegInf : v + 0.0f; }

// Candidate e (larger than every id seen so far in this lane) into the
// lane's top-2; an id of -1 marks an empty slot.
__device__ __forceinline__ void insert_in_order(float v, int e, float& v1, int& i1, float& v2,
                                                int& i2) {
  if (v > v1 || i1 < 0) {
    v2 = v1;
    i2 = i1;
    v1 = v;
    i1 = e;
  } else if (v > v2 || i2 < 0) {
    v2 = v;
    i2 = e;
  }
}

// (v, e) precedes (w, f): larger value, then lower id; empty slots last.
__device__ __forceinline__ bool precedes(float v, int e, float w, int f) {
  if (e < 0) return false;
  if (f < 0) return true;
  return v > w || (v == w && e < f);
}

// Merges the L partial top-2 lists of a row's lane group (xor shuffles; the
// group is L consecutive lanes).
template <int L>
__device__ __forceinline__ void merge_lane_group(float& v1, int& i1, float& v2, int& i2) {
#pragma unroll
  for (int off = L / 2; off > 0; off >>= 1) {
    const float o1 = __shfl_xor_sync(0xffffffffu, v1, off);
    const int p1 = __shfl_xor_sync(0xffffffffu, i1, off);
    const float o2 = __shfl_xor_sync(0xffffffffu, v2, off);
    const int p2 = __shfl_xor_sync(0xffffffffu, i2, off);
    if (precedes(o1, p1, v1, i1)) {
      // The other list's first leads; second is the better of ours and its second.
      if (precedes(v1, i1, o2, p2)) {
        v2 = v1;
        i2 = i1;
      } else {
        v2 = o2;
        i2 = p2;
      }
      v1 = o1;
      i1 = p1;
    } else if (precedes(o1, p1, v2, i2)) {
      v2 = o1;
      i2 = p1;
    }
  }
}

// Weights of a ranked row and the stores of its ids and weights (kPair: one
// 8-byte store each, for 8-byte aligned outputs; chosen at launch, since a
// run-time branch here measured 0.25 us slower per C5 launch).
template <bool kPair>
__device__ __forceinline__ void write_row(long long row, float v1, int i1, float v2, int i2,
                                          int32_t* __restrict__ ids,
                                          float* __restrict__ weights,
                                          const int32_t* __restrict__ remap) {
  int id0 = i1;
  int id1 = i2;
  float w0 = 0.5f, w1 = 0.5f;
  if (v1 != v2) {
    if (v1 == -kNegInf || v2 == kNegInf) {
      w0 = 1.0f;
      w1 = 0.0f;
    } else {
      const float rel = expf(v2 - v1);
      w0 = 1.0f / (1.0f + rel);
      w1 = rel * w0;
    }
  }
  if (remap != nullptr) {
    id0 = __ldg(remap + id0);
    id1 = __ldg(remap + id1);
  }
  if constexpr (kPair) {
    reinterpret_cast<int2*>(ids)[row] = make_int2(id0, id1);
    reinterpret_cast<float2*>(weights)[row] = make_float2(w0, w1);
  } else {
    ids[2 * row] = id0;
    ids[2 * row + 1] = id1;
    weights[2 * row] = w0;
    weights[2 * row + 1] = w1;
  }
}

// Candidate e into a lane top-2 that already holds two valid entries
// (v1, i1) >= (v2, i2), e above every id seen. A strict compare decides
// (a later equal value never precedes an earlier one), and a NaN candidate
// fails both compares, so it needs no canonical form here.
__device__ __forceinline__ void insert_ranked(float v, int e, float& v1, int& i1, float& v2,
                                              int& i2) {
  const bool above1 = v > v1;
  const bool above2 = v > v2;
  const float tv = above2 ? v : v2;
  const int ti = above2 ? e : i2;
  v2 = above1 ? v1 : tv;
  i2 = above1 ? i1 : ti;
  v1 = above1 ? v : v1;
  i1 = above1 ? e : i1;
}

// Candidates of one 16-byte group (experts 4q..4q+3) into the lane's top-2.
// The lane's first group (first == true) seeds the list with its first two
// candidates in canonical form (NaN as -inf), so every later compare sees
// two valid entries; the lower id leads on equal values.
__device__ __forceinline__ void insert4(float4 v, const float* __restrict__ bias, int q,
                                        bool first, float& v1, int& i1, float& v2, int& i2) {
  if (bias != nullptr) {
    const float4 b = __ldg(reinterpret_cast<const float4*>(bias) + q);
    v.x = v.x + b.x;
    v.y = v.y + b.y;
    v.z = v.z + b.z;
    v.w = v.w + b.w;
  }
  const int e = q << 2;
  if (first) {
    const float a = canonical(v.x);
    const float c = canonical(v.y);
    const bool swap = c > a;
    v1 = swap ? c : a;
    i1 = swap ? e + 1 : e;
    v2 = swap ? a : c;
    i2 = swap ? e : e + 1;
  } else {
    insert_ranked(v.x, e, v1, i1, v2, i2);
    insert_ranked(v.y, e + 1, v1, i1, v2, i2);
  }
  insert_ranked(v.z, e + 2, v1, i1, v2, i2);
  insert_ranked(v.w, e + 3, v1, i1, v2, i2);
}

// kPer: 128-bit loads each lane issues before it ranks them (all in flight at
// once); 8 for large batches, 2 for small latency-bound ones. The streaming
// instance (kPer = 8) runs three 256-thread CTAs per SM (at most 85 registers)
// and, before any row is read, has one thread issue an L2 bulk prefetch of
// every row group the CTA will rank: DRAM then streams the whole input while
// the warps rank, and each warp's later groups load from L2. (Measured at
// T=65536, E=128 with bias, one launch in a graph of 50-100: 10.4-10.7 us
// before, 7.9-8.1 us with both; 2, 4 or 5 CTAs per SM, one contiguous chunk
// of groups per CTA, the bias held in registers and register double
// buffering of the next group were each slower.)
template <int L, bool kVec, int kPer, bool kPair, bool kFull>
__global__ void __launch_bounds__(256, kPer == 8 ? 3 : 1)
    topk_gate_kernel(const float* __restrict__ logits, const float* __restrict__ bias,
                     int32_t* __restrict__ ids, float* __restrict__ weights, int tokens,
                     int experts, const int32_t* __restrict__ remap) {
  constexpr int kRowsPerWarp = 32 / L;
  const int lane = threadIdx.x & 31;
  const int group = lane / L;
  const int j = lane % L;
  // This CTA ranks row groups blockIdx.x, blockIdx.x + gridDim.x, ... of
  // rows_per_cta rows each; warp w owns rows w * kRowsPerWarp .. of a group.
  const long long rows_per_cta = static_cast<long long>(blockDim.x >> 5) * kRowsPerWarp;
  const long long cta_stride = static_cast<long long>(gridDim.x) * rows_per_cta;
  const long long lrow = static_cast<long long>(threadIdx.x >> 5) * kRowsPerWarp + group;
  if constexpr (kVec && kPer == 8) {
    // Rows are 16-byte multiples and the base is 16-byte aligned (the kVec
    // conditions), as the bulk prefetch requires.
    if (threadIdx.x == 0) {
      for (long long r0 = blockIdx.x * rows_per_cta; r0 < tokens; r0 += cta_stride) {
        const long long rows = tokens - r0 < rows_per_cta ? tokens - r0 : rows_per_cta;
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(logits + r0 * experts),
                     "r"(static_cast<unsigned>(rows * experts * 4))
                     : "memory");
      }
    }
  }
  for (long long r0 = blockIdx.x * rows_per_cta; r0 < tokens; r0 += cta_stride) {
    const long long row = r0 + lrow;
    const bool active = row < tokens;
    float v1 = kNegInf, v2 = kNegInf;
    int i1 = -1, i2 = -1;
    if (active) {
      const float* src = logits + row * experts;
      if constexpr (kVec && kPer == 8) {
        // One pass: launch_per picks L >= nvec / 8, so the L lanes' 8 loads
        // cover the row. A row of exactly L * 8 groups (kFull) needs no
        // guards; a separate instance, since a run-time choice between the
        // two bodies measured slower.
        const int nvec = experts >> 2;
        const float4* src4 = reinterpret_cast<const float4*>(src);
        float4 v[kPer];
        if constexpr (kFull) {
#pragma unroll
          for (int u = 0; u < kPer; ++u) v[u] = __ldcs(src4 + j + u * L);
#pragma unroll
          for (int u = 0; u < kPer; ++u) insert4(v[u], bias, j + u * L, u == 0, v1, i1, v2, i2);
        } else {
#pragma unroll
          for (int u = 0; u < kPer; ++u) {
            if (j + u * L < nvec) v[u] = __ldcs(src4 + j + u * L);
          }
#pragma unroll
          for (int u = 0; u < kPer; ++u) {
            if (j + u * L < nvec) insert4(v[u], bias, j + u * L, u == 0, v1, i1, v2, i2);
          }
        }
      } else if constexpr (kVec) {
        const int nvec = experts >> 2;
        const float4* src4 = reinterpret_cast<const float4*>(src);
        for (int q0 = j; q0 < nvec; q0 += L * kPer) {
          float4 v[kPer];
#pragma unroll
          for (int u = 0; u < kPer; ++u) {
            const int q = q0 + u * L;
            if (q < nvec) v[u] = __ldcs(src4 + q);
          }
#pragma unroll
          for (int u = 0; u < kPer; ++u) {
            const int q = q0 + u * L;
            if (q < nvec) insert4(v[u], bias, q, u == 0 && q0 == j, v1, i1, v2, i2);
          }
        }
      } else {
#pragma unroll 4
        for (int e = j; e < experts; e += L) {
          float v = __ldg(src + e);
          if (bias != nullptr) v = v + __ldg(bias + e);
          insert_in_order(canonical(v), e, v1, i1, v2, i2);
        }
      }
    }

    merge_lane_group<L>(v1, i1, v2, i2);
    if (!active || j != 0) continue;
    write_row<kPair>(row, v1, i1, v2, i2, ids, weights, remap);
  }
}

template <int L, bool kVec, int kPer, bool kPair, bool kFull>
cudaError_t launch_l(const float* logits, const float* bias, int32_t* ids, float* weights,
                     int tokens, int experts, const int32_t* remap, cudaStream_t stream) {
  constexpr int kThreads = 256;
  constexpr int kRowsPerBlock = (kThreads / 32) * (32 / L);
  // One resident wave (CTAs per SM from the occupancy of this instance).
  static int per_sm = 0;
  if (per_sm == 0) {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, topk_gate_kernel<L, kVec, kPer, kPair, kFull>,
                                                      kThreads, 0) != cudaSuccess || n < 1) {
      cudaGetLastError();
      n = 1;
    }
    per_sm = n;
  }
  const int blocks = min(ceil_div(tokens, kRowsPerBlock), per_sm * sm_count());
  topk_gate_kernel<L, kVec, kPer, kPair, kFull><<<blocks, kThreads, 0, stream>>>(
      logits, bias, ids, weights, tokens, experts, remap);
  note_launch();
  return cudaGetLastError();
}

// Instance by store width and, for the one-pass streaming instance, by
// whether the L lanes' 8 loads exactly cover a row.
template <int L, bool kVec, int kPer>
cudaError_t launch_pf(const float* logits, const float* bias, int32_t* ids, float* weights,
                      int tokens, int experts, bool pair, const int32_t* remap,
                      cudaStream_t stream) {
  if constexpr (kVec && kPer == 8) {
    if ((experts >> 2) == L * kPer) {
      return pair ? launch_l<L, kVec, kPer, true, true>(logits, bias, ids, weights, tokens,
                                                        experts, remap, stream)
                  : launch_l<L, kVec, kPer, false, true>(logits, bias, ids, weights, tokens,
                                                         experts, remap, stream);
    }
  }
  return pair ? launch_l<L, kVec, kPer, true, false>(logits, bias, ids, weights, tokens, experts,
                                                     remap, stream)
              : launch_l<L, kVec, kPer, false, false>(logits, bias, ids, weights, tokens, experts,
                                                      remap, stream);
}

template <bool kVec, int kPer>
cudaError_t launch_per(const float* logits, const float* bias, int32_t* ids, float* weights,
                       int tokens, int experts, bool pair, const int32_t* remap,
                       cudaStream_t stream) {
  // About kPer loads (4 * kPer candidates with 128-bit loads) per lane.
  const int items = kVec ? (experts >> 2) : experts;
  const int per = kVec ? kPer : 4;
  const int want = (items + per - 1) / per;
  int l = 1;
  while (l < want && l < 32) l <<= 1;
  switch (l) {
    case 1: return launch_pf<1, kVec, kPer>(logits, bias, ids, weights, tokens, experts, pair, remap, stream);
    case 2: return launch_pf<2, kVec, kPer>(logits, bias, ids, weights, tokens, experts, pair, remap, stream);
    case 4: return launch_pf<4, kVec, kPer>(logits, bias, ids, weights, tokens, experts, pair, remap, stream);
    case 8: return launch_pf<8, kVec, kPer>(logits, bias, ids, weights, tokens, experts, pair, remap, stream);
    case 16: return launch_pf<16, kVec, kPer>(logits, bias, ids, weights, tokens, experts, pair, remap, stream);
    default: return launch_pf<32, kVec, kPer>(logits, bias, ids, weights, tokens, experts, pair, remap, stream);
  }
}

// Batches from this many rows up stream the logits with 8 loads per lane.
// (A variant that staged rows in shared memory with cp.async.bulk, 192 KB in
// flight per SM, measured slower at C5: 26.7 us with 8 warps per SM and
// 15.1 us with 32, against 10.7 us for the register-staged kernel without
// the L2 prefetch.)
constexpr int kStreamingRows = 16384;

}  // namespace

cudaError_t launch_topk_gate(const float* logits, const float* bias, int32_t* ids, float* weights,
                             int tokens, int experts, cudaStream_t stream, const int32_t* remap) {
  if (tokens <= 0) return cudaSuccess;
  const bool vec = (experts % 4 == 0) && aligned_to(logits, 16) &&
                   (bias == nullptr || aligned_to(bias, 16));
  const bool pair = aligned_to(ids, 8) && aligned_to(weights, 8);
  if (!vec) {
    return launch_per<false, 1>(logits, bias, ids, weights, tokens, experts, pair, remap, stream);
  }
  return tokens >= kStreamingRows
             ? launch_per<true, 8>(logits, bias, ids, weights, tokens, experts, pair, remap, stream)
             : launch_per<true, 2>(logits, bias, ids, weights, tokens, experts, pair, remap, stream);
}

}  // namespace rrb
