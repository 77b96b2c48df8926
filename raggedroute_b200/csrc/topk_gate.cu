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
// stride allows it. Candidates are packed into a 64-bit key
//   (order-preserving bits of the value) << 32 | (~expert id)
// so "precedes" is a plain unsigned comparison: -0 is canonicalised to +0
// first (they compare equal in float), NaN becomes -inf, and the id half
// breaks ties toward the lower id. Each lane keeps its local top-2 keys; the
// group merges them with xor shuffles. The kernel is HBM-bound: 4*E bytes in
// and 16 bytes out per row. An optional remap table rewrites each selected id
// on output (the expert-parallel runtime's replicated "virtual" experts).
#include "common.cuh"

namespace rrb {
namespace {

__device__ __forceinline__ unsigned long long make_key(float raw, int id, bool& non_nan) {
  const bool is_nan = raw != raw;
  non_nan = non_nan || !is_nan;
  float v = is_nan ? -__int_as_float(0x7f800000) : raw + 0.0f;  // -0 -> +0
  const unsigned b = __float_as_uint(v);
  const unsigned ord = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return (static_cast<unsigned long long>(ord) << 32) | static_cast<unsigned>(0xffffffffu - id);
}

__device__ __forceinline__ float key_value(unsigned long long key) {
  const unsigned ord = static_cast<unsigned>(key >> 32);
  const unsigned b = (ord & 0x80000000u) ? (ord & 0x7fffffffu) : ~ord;
  return __uint_as_float(b);
}

__device__ __forceinline__ int key_id(unsigned long long key) {
  return static_cast<int>(0xffffffffu - static_cast<unsigned>(key));
}

__device__ __forceinline__ void insert(unsigned long long key, unsigned long long& k1,
                                       unsigned long long& k2) {
  if (key > k1) {
    k2 = k1;
    k1 = key;
  } else if (key > k2) {
    k2 = key;
  }
}

// kPer: 128-bit loads each lane issues before it ranks them (all in flight at
// once); 8 for large batches so that one wave of CTAs keeps enough bytes in
// flight to stream the logits at HBM speed, 2 for small latency-bound ones.
template <int L, bool kVec, int kPer>
__global__ void __launch_bounds__(256) topk_gate_kernel(const float* __restrict__ logits,
                                                        const float* __restrict__ bias,
                                                        int32_t* __restrict__ ids,
                                                        float* __restrict__ weights, int tokens,
                                                        int experts, bool pair_stores,
                                                        const int32_t* __restrict__ remap) {
  constexpr int kRowsPerWarp = 32 / L;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int group = lane / L;
  const int j = lane % L;
  const long long row = (static_cast<long long>(blockIdx.x) * (blockDim.x >> 5) + warp) *
                            kRowsPerWarp + group;
  const bool active = row < tokens;

  unsigned long long k1 = 0, k2 = 0;
  bool non_nan = false;
  if (active) {
    const float* src = logits + row * experts;
    if constexpr (kVec) {
      const int nvec = experts >> 2;
      const float4* src4 = reinterpret_cast<const float4*>(src);
      const float4* bias4 = reinterpret_cast<const float4*>(bias);
      // Keys order candidates totally (value, then lower id), so the order
      // in which a lane ranks its candidates does not change the result.
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
          if (q < nvec) {
            if (bias != nullptr) {
              const float4 b = __ldg(bias4 + q);
              v[u].x = v[u].x + b.x;
              v[u].y = v[u].y + b.y;
              v[u].z = v[u].z + b.z;
              v[u].w = v[u].w + b.w;
            }
            const int e = q << 2;
            insert(make_key(v[u].x, e, non_nan), k1, k2);
            insert(make_key(v[u].y, e + 1, non_nan), k1, k2);
            insert(make_key(v[u].z, e + 2, non_nan), k1, k2);
            insert(make_key(v[u].w, e + 3, non_nan), k1, k2);
          }
        }
      }
    } else {
#pragma unroll 4
      for (int e = j; e < experts; e += L) {
        float v = __ldg(src + e);
        if (bias != nullptr) v = v + __ldg(bias + e);
        insert(make_key(v, e, non_nan), k1, k2);
      }
    }
  }

  // Merge the L partial top-2 lists of this row's lane group.
#pragma unroll
  for (int off = L / 2; off > 0; off >>= 1) {
    const unsigned long long o1 = __shfl_xor_sync(0xffffffffu, k1, off);
    const unsigned long long o2 = __shfl_xor_sync(0xffffffffu, k2, off);
    const bool o_nan = __shfl_xor_sync(0xffffffffu, non_nan ? 1 : 0, off) != 0;
    non_nan = non_nan || o_nan;
    if (o1 > k1) {
      k2 = (k1 > o2) ? k1 : o2;
      k1 = o1;
    } else {
      k2 = (o1 > k2) ? o1 : k2;
    }
  }

  if (!active || j != 0) return;
  int id0 = key_id(k1);
  int id1 = key_id(k2);
  const float v0 = key_value(k1);
  const float v1 = key_value(k2);
  float w0 = 0.5f, w1 = 0.5f;
  if (!non_nan) {
    id0 = 0;
    id1 = 1;
  } else if (v0 != v1) {
    if (v0 == __int_as_float(0x7f800000) || v1 == -__int_as_float(0x7f800000)) {
      w0 = 1.0f;
      w1 = 0.0f;
    } else {
      const float rel = expf(v1 - v0);
      w0 = 1.0f / (1.0f + rel);
      w1 = rel * w0;
    }
  }
  if (remap != nullptr) {
    id0 = __ldg(remap + id0);
    id1 = __ldg(remap + id1);
  }
  if (pair_stores) {
    reinterpret_cast<int2*>(ids)[row] = make_int2(id0, id1);
    reinterpret_cast<float2*>(weights)[row] = make_float2(w0, w1);
  } else {
    ids[2 * row] = id0;
    ids[2 * row + 1] = id1;
    weights[2 * row] = w0;
    weights[2 * row + 1] = w1;
  }
}

template <int L, bool kVec, int kPer>
cudaError_t launch_l(const float* logits, const float* bias, int32_t* ids, float* weights,
                     int tokens, int experts, bool pair, const int32_t* remap,
                     cudaStream_t stream) {
  constexpr int kThreads = 256;
  constexpr int kRowsPerBlock = (kThreads / 32) * (32 / L);
  const int blocks = ceil_div(tokens, kRowsPerBlock);
  topk_gate_kernel<L, kVec, kPer><<<blocks, kThreads, 0, stream>>>(
      logits, bias, ids, weights, tokens, experts, pair, remap);
  note_launch();
  return cudaGetLastError();
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
    case 1: return launch_l<1, kVec, kPer>(logits, bias, ids, weights, tokens, experts, pair, remap, stream);
    case 2: return launch_l<2, kVec, kPer>(logits, bias, ids, weights, tokens, experts, pair, remap, stream);
    case 4: return launch_l<4, kVec, kPer>(logits, bias, ids, weights, tokens, experts, pair, remap, stream);
    case 8: return launch_l<8, kVec, kPer>(logits, bias, ids, weights, tokens, experts, pair, remap, stream);
    case 16: return launch_l<16, kVec, kPer>(logits, bias, ids, weights, tokens, experts, pair, remap, stream);
    default: return launch_l<32, kVec, kPer>(logits, bias, ids, weights, tokens, experts, pair, remap, stream);
  }
}

// Batches from this many rows up stream the logits with 8 loads per lane.
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
