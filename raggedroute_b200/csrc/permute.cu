// Stable token permute for B200.
//
// Contract (src/permute/operator.cpp:22-83 and src/permute/cpu_reference/
// reference.cpp:22-81 of the reference, with the slot order made
// deterministic): for route r = t*top_k + k with expert e = ids[r],
//   route_pos[r] = offsets[e] + #{r' < r : ids[r'] == e}
//   x_permuted[route_pos[r], :] = x[t, :]        (bit-exact copy)
//   sorted_route[route_pos[r]] = r               (optional)
//   cursors[e] == #{r : ids[r] == e} afterwards  (the reference's post-state)
// The reference assigns slots with an atomic cursor, so its order varies run
// to run; the route-ascending order used here is the unique order that a
// sequential counting sort produces and passes every reference set check.
//
// Design (no atomics on positions, so the result never depends on
// scheduling): routes are cut into token-aligned chunks, one CTA each.
//   1. count:  per-chunk expert histogram -> the chunk's row of the chunk
//              table (below).
//   2. scan:   column-wise exclusive scan over chunks, seeded with offsets,
//              giving each chunk its first slot per expert, in place.
//   3. place:  inside a chunk each warp owns a contiguous run of routes; the
//              per-(warp, expert) counts are scanned in shared memory and the
//              rank inside a warp step is the popcount of the lower lanes with
//              the same expert. The lanes with the same expert come from one
//              ballot per bit of the expert id, a cost that does not grow with
//              the number of distinct experts in a warp (__match_any_sync's
//              does: measured in the histogram, 1M uniform routes took 14.4 us
//              over 256 experts against 6.2 us over one). The CTA then copies
//              each token row once from x (128-bit loads) to its top_k
//              destinations.
// A single chunk needs neither step 1 nor 2. The only workspace is the
// reference's E int32 cursors (src/permute/operator.cpp:17-19), for every
// input size: every chunk but the last spans at least E routes and keeps its
// row of the chunk table (E int32) in the first E entries of its own slice
// of route_pos, which the place step reads before it overwrites that slice
// with the route positions; the last chunk keeps its row in the cursors,
// which the place step then overwrites with the per-expert counts (the
// reference's post-state). No chunk reads or writes another's slice. HBM
// traffic is the algorithmic minimum: x read once, x_permuted written once,
// ids read three times (4 bytes per route each).
#include "common.cuh"

namespace rrb {
namespace {

constexpr int kPlaceThreads = 256;
constexpr int kPlaceWarps = kPlaceThreads / 32;
constexpr int kMaxChunkRoutes = 4096;
constexpr int kMaxPerLane = kMaxChunkRoutes / kPlaceThreads;  // 16
// About one resident wave of place CTAs (8 per SM): the copy work of a chunk
// is proportional to its tokens, so with ~7 chunks per SM the busiest SM
// carries ~1% more than the mean (512 chunks, 3.46 per SM, cost 16%).
constexpr int kTargetChunks = 8 * kNumSms;

struct ChunkPlan {
  int tokens_per_chunk;
  int chunks;
};

ChunkPlan plan_chunks(int tokens, int top_k, int experts) {
  const long long routes = static_cast<long long>(tokens) * top_k;
  long long want = (routes + kTargetChunks - 1) / kTargetChunks;
  long long rc = 128;
  while (rc < want && rc < kMaxChunkRoutes) rc <<= 1;
  // A chunk's table row lives in its own slice of route_pos: >= E routes
  // (E <= 1024 keeps this within kMaxChunkRoutes).
  while (rc < experts) rc <<= 1;
  int tc = static_cast<int>(rc / top_k);
  if (tc < 1) tc = 1;
  if (static_cast<long long>(tc) * top_k < experts) tc = ceil_div(experts, top_k);
  ChunkPlan p;
  p.tokens_per_chunk = tc;
  p.chunks = tokens <= 0 ? 0 : ceil_div(tokens, tc);
  return p;
}

__device__ __forceinline__ int warp_leader(unsigned peers) { return __ffs(peers) - 1; }

// Bits of the keys 0..max_key.
__device__ __forceinline__ int key_bits(int max_key) { return max_key <= 0 ? 0 : 32 - __clz(max_key); }

// The lanes of the warp whose key equals this lane's (keys in [0, 2^nbits),
// nbits warp-uniform; all 32 lanes call it): one ballot per key bit.
__device__ __forceinline__ unsigned same_key_lanes(unsigned key, int nbits) {
  unsigned m = 0xffffffffu;
  for (int b = 0; b < nbits; ++b) {
    const bool bit = (key >> b) & 1u;
    const unsigned bal = __ballot_sync(0xffffffffu, bit);
    m &= bit ? bal : ~bal;
  }
  return m;
}

// Row c of the chunk table: the first E entries of chunk c's slice of
// route_pos, or the cursors for the last chunk.
__device__ __forceinline__ int32_t* chunk_row(int32_t* route_pos, int32_t* cursors, int c,
                                              int chunks, int routes_per_chunk) {
  return c == chunks - 1 ? cursors
                         : route_pos + static_cast<long long>(c) * routes_per_chunk;
}

// Per-chunk histogram into the chunk's table row.
__global__ void __launch_bounds__(kPlaceThreads) permute_count_kernel(
    const int32_t* __restrict__ ids, int routes, int experts, int routes_per_chunk,
    int32_t* route_pos, int32_t* cursors) {
  extern __shared__ int hist[];
  for (int i = threadIdx.x; i < experts; i += blockDim.x) hist[i] = 0;
  __syncthreads();
  const long long r0 = static_cast<long long>(blockIdx.x) * routes_per_chunk;
  long long r1 = r0 + routes_per_chunk;
  if (r1 > routes) r1 = routes;
  const int lane = threadIdx.x & 31;
  const int nbits = key_bits(experts);
  for (long long base = r0 + (threadIdx.x & ~31); base < r1; base += blockDim.x) {
    const long long r = base + lane;
    const int e = r < r1 ? __ldg(ids + r) : -1;
    const bool valid = e >= 0 && e < experts;
    // Key 0 gathers every id outside the contract (never counted).
    const unsigned peers = same_key_lanes(valid ? e + 1 : 0, nbits);
    if (lane == warp_leader(peers) && valid) atomicAdd(hist + e, __popc(peers));
  }
  __syncthreads();
  int32_t* row = chunk_row(route_pos, cursors, blockIdx.x, gridDim.x, routes_per_chunk);
  for (int i = threadIdx.x; i < experts; i += blockDim.x) row[i] = hist[i];
}

// Column-wise exclusive scan over the chunk table, in place, seeded with
// offsets. Each CTA owns 32 experts (one per lane); its 32 warps split the
// chunk range. Up to kKeep chunks per warp (chunk tables up to 1280 rows,
// which covers every input up to 5.2M routes) the column is loaded once, all
// loads in flight together, kept in registers and written back scanned; larger
// tables take two batched passes.
constexpr int kScanKeep = 40;

template <bool kKeep>
__global__ void __launch_bounds__(1024) permute_scan_kernel(int32_t* route_pos, int32_t* cursors,
                                                            const int32_t* __restrict__ offsets,
                                                            int chunks, int routes_per_chunk,
                                                            int experts) {
  __shared__ int part[32][33];
  const int lane = threadIdx.x & 31;
  const int grp = threadIdx.x >> 5;
  const int e = blockIdx.x * 32 + lane;
  const int per = (chunks + 31) / 32;
  const int c0 = grp * per;
  const int c1 = min(chunks, c0 + per);
  constexpr int kBatch = 8;  // loads in flight per lane on the two-pass path
  auto row = [&](int c) { return chunk_row(route_pos, cursors, c, chunks, routes_per_chunk); };
  int keep[kKeep ? kScanKeep : 1];
  int sum = 0;
  if (e < experts) {
    if constexpr (kKeep) {
#pragma unroll
      for (int u = 0; u < kScanKeep; ++u) {
        keep[u] = c0 + u < c1 ? row(c0 + u)[e] : 0;
      }
#pragma unroll
      for (int u = 0; u < kScanKeep; ++u) sum += keep[u];
    } else {
      for (int c = c0; c < c1; c += kBatch) {
        int v[kBatch];
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
          v[u] = c + u < c1 ? row(c + u)[e] : 0;
        }
#pragma unroll
        for (int u = 0; u < kBatch; ++u) sum += v[u];
      }
    }
  }
  part[grp][lane] = sum;
  __syncthreads();
  if (grp == 0) {
    int run = 0;
    for (int g = 0; g < 32; ++g) {
      const int v = part[g][lane];
      part[g][lane] = run;
      run += v;
    }
  }
  __syncthreads();
  if (e < experts) {
    int run = offsets[e] + part[grp][lane];
    if constexpr (kKeep) {
#pragma unroll
      for (int u = 0; u < kScanKeep; ++u) {
        if (c0 + u < c1) row(c0 + u)[e] = run;
        run += keep[u];
      }
    } else {
      for (int c = c0; c < c1; c += kBatch) {
        int v[kBatch];
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
          v[u] = c + u < c1 ? row(c + u)[e] : 0;
        }
#pragma unroll
        for (int u = 0; u < kBatch; ++u) {
          if (c + u < c1) row(c + u)[e] = run;
          run += v[u];
        }
      }
    }
  }
}

// Copy a row of `hidden` floats from src to top_k destinations; one warp.
template <bool kVec>
__device__ __forceinline__ void copy_row_warp(const float* __restrict__ src, float* __restrict__ xp,
                                              const int* dest, int top_k, int hidden) {
  const int lane = threadIdx.x & 31;
  if constexpr (kVec) {
    const int n4 = hidden >> 2;
    const float4* s4 = reinterpret_cast<const float4*>(src);
    int i = lane;
    for (; i + 96 < n4; i += 128) {
      const float4 a = __ldg(s4 + i);
      const float4 b = __ldg(s4 + i + 32);
      const float4 c = __ldg(s4 + i + 64);
      const float4 d = __ldg(s4 + i + 96);
      for (int k = 0; k < top_k; ++k) {
        if (dest[k] < 0) continue;
        float4* d4 = reinterpret_cast<float4*>(xp + static_cast<long long>(dest[k]) * hidden);
        __stcs(d4 + i, a);
        __stcs(d4 + i + 32, b);
        __stcs(d4 + i + 64, c);
        __stcs(d4 + i + 96, d);
      }
    }
    for (; i < n4; i += 32) {
      const float4 a = __ldg(s4 + i);
      for (int k = 0; k < top_k; ++k) {
        if (dest[k] < 0) continue;
        float4* d4 = reinterpret_cast<float4*>(xp + static_cast<long long>(dest[k]) * hidden);
        __stcs(d4 + i, a);
      }
    }
  } else {
    for (int i = lane; i < hidden; i += 32) {
      const float a = __ldg(src + i);
      for (int k = 0; k < top_k; ++k) {
        if (dest[k] < 0) continue;
        xp[static_cast<long long>(dest[k]) * hidden + i] = a;
      }
    }
  }
}

// Copy a row to up to 8 destination rows given as pointers (nullptr = skip);
// the destinations may be another rank's memory. One warp.
template <bool kVec>
__device__ __forceinline__ void copy_row_warp_to(const float* __restrict__ src, float* const* dst,
                                                 int n, int hidden) {
  const int lane = threadIdx.x & 31;
  if constexpr (kVec) {
    const int n4 = hidden >> 2;
    const float4* s4 = reinterpret_cast<const float4*>(src);
    int i = lane;
    for (; i + 96 < n4; i += 128) {
      const float4 a = __ldg(s4 + i);
      const float4 b = __ldg(s4 + i + 32);
      const float4 c = __ldg(s4 + i + 64);
      const float4 d = __ldg(s4 + i + 96);
      for (int k = 0; k < n; ++k) {
        if (dst[k] == nullptr) continue;
        float4* d4 = reinterpret_cast<float4*>(dst[k]);
        d4[i] = a;
        d4[i + 32] = b;
        d4[i + 64] = c;
        d4[i + 96] = d;
      }
    }
    for (; i < n4; i += 32) {
      const float4 a = __ldg(s4 + i);
      for (int k = 0; k < n; ++k) {
        if (dst[k] != nullptr) reinterpret_cast<float4*>(dst[k])[i] = a;
      }
    }
  } else {
    for (int i = lane; i < hidden; i += 32) {
      const float a = __ldg(src + i);
      for (int k = 0; k < n; ++k) {
        if (dst[k] != nullptr) dst[k][i] = a;
      }
    }
  }
}

// Place + copy of one chunk. With one chunk the slots are seeded by offsets;
// with several, by the chunk's row of the scanned chunk table. The single or
// last chunk writes the cursor post-state (per-expert counts).
// With kPeer the rows go to the owners' receive buffers (PeerDispatch) and
// xp / sorted_route are unused; only routes whose local expert index
// (expert % local) lies in [peer.le_lo, peer.le_hi) are sent, so a dispatch
// can be split into launches over expert ranges (route_pos is written in
// full by every launch, with the same values).
template <bool kVec, bool kPeer>
__device__ __forceinline__ void place_chunk(
    int chunk, int chunks, int* smem, const int& aborted, const float* __restrict__ x,
    const int32_t* __restrict__ ids, const int32_t* __restrict__ offsets, float* __restrict__ xp,
    int32_t* route_pos, int32_t* __restrict__ sorted_route, int32_t* cursors, int tokens,
    int experts, int top_k, int hidden, int tokens_per_chunk, const PeerDispatch& peer) {
  int* warp_base = smem;                            // [kPlaceWarps][experts]
  int* pos = smem + kPlaceWarps * experts;          // [routes in chunk]
  // Peer mode: packed (owner << 40 | receive row) per route, -1 = dropped.
  long long* remote = reinterpret_cast<long long*>(
      smem + ((kPlaceWarps * experts + kMaxChunkRoutes + 1) & ~1));
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int t0 = chunk * tokens_per_chunk;
  const int t1 = min(tokens, t0 + tokens_per_chunk);
  const long long r0 = static_cast<long long>(t0) * top_k;
  const int nr = (t1 - t0) * top_k;
  // Each warp owns a contiguous run of `per_warp` routes (a multiple of 32).
  const int per_warp = ((nr + kPlaceWarps - 1) / kPlaceWarps + 31) & ~31;
  const int w0 = warp * per_warp;
  const int steps = per_warp >> 5;  // <= kMaxPerLane

  for (int i = threadIdx.x; i < kPlaceWarps * experts; i += blockDim.x) warp_base[i] = 0;
  __syncthreads();

  // Pass 1: per-warp expert counts; ids stay in registers. Keys: expert + 1,
  // 0 for "no route" and "out of contract".
  const int nbits = key_bits(experts);
  int my_ids[kMaxPerLane];
  int* my_count = warp_base + warp * experts;
#pragma unroll
  for (int s = 0; s < kMaxPerLane; ++s) {
    my_ids[s] = -1;
    if (s < steps) {
      const int local = w0 + s * 32 + lane;
      int e = -1;
      if (local < nr) {
        e = __ldg(ids + r0 + local);
        if (e < 0 || e >= experts) e = -2;  // out of contract: skipped
      }
      my_ids[s] = e;
      const unsigned peers = same_key_lanes(e >= 0 ? e + 1 : 0, nbits);
      if (lane == warp_leader(peers) && e >= 0) my_count[e] += __popc(peers);
      __syncwarp();
    }
  }
  __syncthreads();

  // Per-(warp, expert) starting slots, from the chunk's table row (read
  // here, before pass 2 overwrites this chunk's slice of route_pos).
  const bool chunked = chunks > 1;
  const bool last = chunk == chunks - 1;
  const int32_t* row =
      chunked ? chunk_row(route_pos, cursors, chunk, chunks, tokens_per_chunk * top_k) : offsets;
  for (int e = threadIdx.x; e < experts; e += blockDim.x) {
    int run = row[e];
#pragma unroll
    for (int w = 0; w < kPlaceWarps; ++w) {
      const int v = warp_base[w * experts + e];
      warp_base[w * experts + e] = run;
      run += v;
    }
    if (last) cursors[e] = run - offsets[e];
  }
  __syncthreads();

  // Pass 2: stable ranks.
  const unsigned lt = lanemask_lt();
#pragma unroll
  for (int s = 0; s < kMaxPerLane; ++s) {
    if (s < steps) {
      const int e = my_ids[s];
      const unsigned peers = same_key_lanes(e >= 0 ? e + 1 : 0, nbits);
      int p = -1;
      if (e >= 0) p = my_count[e] + __popc(peers & lt);
      __syncwarp();
      if (e >= 0 && lane == warp_leader(peers)) my_count[e] += __popc(peers);
      __syncwarp();
      const int local = w0 + s * 32 + lane;
      if (local < nr && e != -1) {
        pos[local] = p;
        route_pos[r0 + local] = p;
        if constexpr (kPeer) {
          long long packed = -1;
          const int le = e >= 0 ? e % peer.local : -1;
          if (p >= 0 && !aborted && le >= peer.le_lo && le < peer.le_hi) {
            const int owner = e / peer.local;
            const long long row = static_cast<long long>(__ldg(peer.dest_off + e)) +
                                  (p - __ldg(offsets + e));
            if (row < peer.capacity) {
              peer.ret_base[owner][row] =
                  (static_cast<long long>(peer.me) << kPeerRankShift) | static_cast<long long>(p);
              packed = (static_cast<long long>(owner) << kPeerRankShift) | row;
            } else {
              raise_device_error(peer.err, kErrEpCapacity);
            }
          }
          remote[local] = packed;
        } else {
          if (sorted_route != nullptr && p >= 0) {
            sorted_route[p] = static_cast<int32_t>(r0 + local);
          }
        }
      }
    }
  }
  __syncthreads();

  if constexpr (kPeer) {
    for (int t = t0 + warp; t < t1; t += kPlaceWarps) {
      const long long* d = remote + static_cast<long long>(t - t0) * top_k;
      for (int k0 = 0; k0 < top_k; k0 += 8) {
        const int kn = min(8, top_k - k0);
        float* dst[8];
        for (int k = 0; k < kn; ++k) {
          const long long v = d[k0 + k];
          dst[k] = v < 0 ? nullptr
                         : peer.x_base[v >> kPeerRankShift] + (v & kPeerRowMask) * hidden;
        }
        copy_row_warp_to<kVec>(x + static_cast<long long>(t) * hidden, dst, kn, hidden);
      }
    }
    return;
  }
  if (hidden <= 0) return;
  if constexpr (kVec) {
    const int n4 = hidden >> 2;
    if (n4 <= 32 && top_k <= 8) {
      // Short rows (hidden <= 128): one 16-byte chunk per lane and row, four
      // rows per warp step, so every lane keeps four loads in flight.
      constexpr int kRows = 4;
      for (int t = t0 + warp; t < t1; t += kRows * kPlaceWarps) {
        float4 v[kRows];
#pragma unroll
        for (int u = 0; u < kRows; ++u) {
          const int tu = t + u * kPlaceWarps;
          if (tu < t1 && lane < n4) {
            v[u] = __ldg(reinterpret_cast<const float4*>(x + static_cast<long long>(tu) * hidden) +
                         lane);
          }
        }
#pragma unroll
        for (int u = 0; u < kRows; ++u) {
          const int tu = t + u * kPlaceWarps;
          if (tu < t1 && lane < n4) {
            const int* d = pos + (tu - t0) * top_k;
            for (int k = 0; k < top_k; ++k) {
              const int dk = d[k];
              if (dk >= 0) {
                __stcs(reinterpret_cast<float4*>(xp + static_cast<long long>(dk) * hidden) + lane,
                       v[u]);
              }
            }
          }
        }
      }
      return;
    }
  }
  // Copy: one warp per token row, read once, written top_k times.
  for (int t = t0 + warp; t < t1; t += kPlaceWarps) {
    int dest[8];
    const int* d = pos + (t - t0) * top_k;
    if (top_k <= 8) {
      for (int k = 0; k < top_k; ++k) dest[k] = d[k];
      copy_row_warp<kVec>(x + static_cast<long long>(t) * hidden, xp, dest, top_k, hidden);
    } else {
      for (int k0 = 0; k0 < top_k; k0 += 8) {
        const int kn = min(8, top_k - k0);
        for (int k = 0; k < kn; ++k) dest[k] = d[k0 + k];
        copy_row_warp<kVec>(x + static_cast<long long>(t) * hidden, xp, dest, kn, hidden);
      }
    }
  }
}

// ---- workspace-free path for the low-level launcher -----------------------

// One CTA: finds the largest expert id, mirrors the caller's cursors into
// shared memory, and ranks every route in order with a single warp. Slot =
// offsets[e] + cursors[e] (running). Cursors are written back at the end.
template <bool kVec, bool kPeer>
__global__ void __launch_bounds__(kPlaceThreads) permute_place_kernel(
    const float* __restrict__ x, const int32_t* __restrict__ ids,
    const int32_t* __restrict__ offsets, float* __restrict__ xp, int32_t* route_pos,
    int32_t* __restrict__ sorted_route, int32_t* cursors, int tokens, int experts, int top_k,
    int hidden, int tokens_per_chunk, int chunks, const PeerDispatch peer) {
  extern __shared__ int smem[];
  __shared__ int aborted;
  if (threadIdx.x == 0) aborted = (kPeer && peer.abort != nullptr) ? *peer.abort : 0;
  // One chunk per CTA (the loop covers a grid smaller than the plan).
  for (int c = blockIdx.x; c < chunks; c += gridDim.x) {
    place_chunk<kVec, kPeer>(c, chunks, smem, aborted, x, ids, offsets, xp, route_pos,
                             sorted_route, cursors, tokens, experts, top_k, hidden,
                             tokens_per_chunk, peer);
    __syncthreads();  // the next chunk reuses the shared memory
  }
  // Peer mode: complete this thread's stores to other ranks' memory before
  // the kernel ends (the barrier that follows then publishes them).
  if constexpr (kPeer) __threadfence_system();
}

// The rest of a split expert-parallel dispatch: every route whose local
// expert index (expert % local) lies in [peer.le_lo, peer.le_hi) is sent to
// its owner at the position the permute already wrote to route_pos (so no
// ranking here), with its return address. One warp per token, grid-stride,
// meant for a few CTAs beside the grouped GEMM. top_k <= 8.
constexpr int kRestThreads = 1024;
// Dynamic shared memory each CTA asks for (unused): more than half an SM's,
// so no two CTAs of this kernel, and no GEMM CTA, share an SM.
constexpr int kRestSmem = 120 * 1024;

template <bool kVec>
__global__ void __launch_bounds__(kRestThreads) ep_dispatch_rest_kernel(
    const float* __restrict__ x, const int32_t* __restrict__ ids,
    const int32_t* __restrict__ offsets, const int32_t* __restrict__ route_pos, int tokens,
    int experts, int top_k, int hidden, const PeerDispatch peer) {
  __shared__ int aborted;
  if (threadIdx.x == 0) aborted = peer.abort != nullptr ? *peer.abort : 0;
  __syncthreads();
  if (aborted) return;
  const int lane = threadIdx.x & 31;
  const long long warp = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const long long nwarps = (static_cast<long long>(gridDim.x) * blockDim.x) >> 5;
  for (long long t = warp; t < tokens; t += nwarps) {
    float* dst[8];
    for (int k = 0; k < top_k; ++k) {
      dst[k] = nullptr;
      const long long r = t * top_k + k;
      const int e = __ldg(ids + r);
      if (e < 0 || e >= experts) continue;
      const int le = e % peer.local;
      if (le < peer.le_lo || le >= peer.le_hi) continue;
      const int p = __ldg(route_pos + r);
      const int owner = e / peer.local;
      const long long row =
          static_cast<long long>(__ldg(peer.dest_off + e)) + (p - __ldg(offsets + e));
      if (row >= peer.capacity) {
        if (lane == 0) raise_device_error(peer.err, kErrEpCapacity);
        continue;
      }
      if (lane == 0) {
        peer.ret_base[owner][row] =
            (static_cast<long long>(peer.me) << kPeerRankShift) | static_cast<long long>(p);
      }
      dst[k] = peer.x_base[owner] + row * hidden;
    }
    copy_row_warp_to<kVec>(x + t * hidden, dst, top_k, hidden);
  }
  // Complete this thread's stores to other ranks' memory before the kernel
  // ends (the barrier that follows then publishes them).
  __threadfence_system();
}

__global__ void __launch_bounds__(1024) permute_cursor_rank_kernel(
    const int32_t* __restrict__ ids, const int32_t* __restrict__ offsets, int32_t* cursors,
    int32_t* __restrict__ route_pos, int32_t* __restrict__ sorted_route, int routes) {
  __shared__ int cur[kMaxExperts];
  __shared__ int max_id;
  if (threadIdx.x == 0) max_id = -1;
  __syncthreads();
  int local_max = -1;
  for (int r = threadIdx.x; r < routes; r += blockDim.x) {
    const int e = __ldg(ids + r);
    if (e >= 0 && e < kMaxExperts && e > local_max) local_max = e;
  }
  atomicMax(&max_id, local_max);
  __syncthreads();
  const int ne = max_id + 1;
  for (int e = threadIdx.x; e < ne; e += blockDim.x) cur[e] = cursors[e];
  __syncthreads();
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    const unsigned lt = lanemask_lt();
    const int nbits = key_bits(kMaxExperts);
    for (int base = 0; base < routes; base += 32) {
      const int r = base + lane;
      int e = r < routes ? __ldg(ids + r) : -1;
      if (e >= kMaxExperts) e = -2;
      const unsigned peers = same_key_lanes(e >= 0 ? e + 1 : 0, nbits);
      int p = -1;
      if (e >= 0) p = offsets[e] + cur[e] + __popc(peers & lt);
      __syncwarp();
      if (e >= 0 && lane == warp_leader(peers)) cur[e] += __popc(peers);
      __syncwarp();
      if (r < routes) {
        route_pos[r] = p;
        if (sorted_route != nullptr && p >= 0) sorted_route[p] = r;
      }
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < ne; e += blockDim.x) cursors[e] = cur[e];
}

template <bool kVec>
__global__ void __launch_bounds__(256) permute_copy_kernel(const float* __restrict__ x,
                                                           const int32_t* __restrict__ route_pos,
                                                           float* __restrict__ xp, int tokens,
                                                           int top_k, int hidden) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int nwarps = (gridDim.x * blockDim.x) >> 5;
  for (int t = warp; t < tokens; t += nwarps) {
    for (int k0 = 0; k0 < top_k; k0 += 8) {
      int dest[8];
      const int kn = min(8, top_k - k0);
      for (int k = 0; k < kn; ++k) dest[k] = route_pos[static_cast<long long>(t) * top_k + k0 + k];
      copy_row_warp<kVec>(x + static_cast<long long>(t) * hidden, xp, dest, kn, hidden);
    }
  }
}

}  // namespace

std::size_t permute_workspace_bytes(int, int experts, int) {
  return experts <= 0 ? 0 : static_cast<std::size_t>(experts) * sizeof(int32_t);
}

namespace {

template <bool kPeer>
cudaError_t permute_impl(const float* x, const int32_t* ids, const int32_t* offsets,
                         float* x_permuted, int32_t* route_pos, int32_t* sorted_route, int tokens,
                         int experts, int top_k, int hidden, void* workspace,
                         const PeerDispatch& peer, cudaStream_t stream) {
  if (tokens <= 0) return cudaSuccess;
  const ChunkPlan p = plan_chunks(tokens, top_k, experts);
  int32_t* cursors = static_cast<int32_t*>(workspace);
  const int routes_per_chunk = p.tokens_per_chunk * top_k;
  const int routes = tokens * top_k;
  if (p.chunks > 1) {
    permute_count_kernel<<<p.chunks, kPlaceThreads, experts * sizeof(int), stream>>>(
        ids, routes, experts, routes_per_chunk, route_pos, cursors);
    if (p.chunks <= 32 * kScanKeep) {
      permute_scan_kernel<true><<<ceil_div(experts, 32), 1024, 0, stream>>>(
          route_pos, cursors, offsets, p.chunks, routes_per_chunk, experts);
    } else {
      permute_scan_kernel<false><<<ceil_div(experts, 32), 1024, 0, stream>>>(
          route_pos, cursors, offsets, p.chunks, routes_per_chunk, experts);
    }
    note_launch(2);
  }
  // Peer mode keeps pos[] at its full size so the int64 table that follows is
  // at a fixed, 8-byte aligned offset.
  const std::size_t ints = static_cast<std::size_t>(kPlaceWarps) * experts +
                           (kPeer ? kMaxChunkRoutes + 1 : routes_per_chunk);
  const std::size_t smem = kPeer ? ((ints & ~static_cast<std::size_t>(1)) * sizeof(int) +
                                    static_cast<std::size_t>(kMaxChunkRoutes) * sizeof(long long))
                                 : ints * sizeof(int);
  const bool vec = hidden % 4 == 0 && aligned_to(x, 16) &&
                   (kPeer || aligned_to(x_permuted, 16));
  if (smem > 48 * 1024) {
    cudaError_t e1 = cudaFuncSetAttribute(permute_place_kernel<true, kPeer>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>(smem));
    cudaError_t e2 = cudaFuncSetAttribute(permute_place_kernel<false, kPeer>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>(smem));
    if (e1 != cudaSuccess) return e1;
    if (e2 != cudaSuccess) return e2;
  }
  if (vec) {
    permute_place_kernel<true, kPeer><<<p.chunks, kPlaceThreads, smem, stream>>>(
        x, ids, offsets, x_permuted, route_pos, sorted_route, cursors, tokens, experts, top_k,
        hidden, p.tokens_per_chunk, p.chunks, peer);
  } else {
    permute_place_kernel<false, kPeer><<<p.chunks, kPlaceThreads, smem, stream>>>(
        x, ids, offsets, x_permuted, route_pos, sorted_route, cursors, tokens, experts, top_k,
        hidden, p.tokens_per_chunk, p.chunks, peer);
  }
  note_launch();
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_token_permute(const float* x, const int32_t* ids, const int32_t* offsets,
                                 float* x_permuted, int32_t* route_pos, int32_t* sorted_route,
                                 int tokens, int experts, int top_k, int hidden, void* workspace,
                                 cudaStream_t stream) {
  return permute_impl<false>(x, ids, offsets, x_permuted, route_pos, sorted_route, tokens,
                             experts, top_k, hidden, workspace, PeerDispatch{}, stream);
}

cudaError_t launch_token_permute_peer(const float* x, const int32_t* ids, const int32_t* offsets,
                                      int32_t* route_pos, int tokens, int experts, int top_k,
                                      int hidden, void* workspace, const PeerDispatch& peer,
                                      cudaStream_t stream) {
  if (peer.x_base == nullptr || peer.ret_base == nullptr || peer.dest_off == nullptr ||
      peer.local < 1) {
    return cudaErrorInvalidValue;
  }
  return permute_impl<true>(x, ids, offsets, nullptr, route_pos, nullptr, tokens, experts, top_k,
                            hidden, workspace, peer, stream);
}

cudaError_t launch_ep_dispatch_rest(const float* x, const int32_t* ids, const int32_t* offsets,
                                    const int32_t* route_pos, int tokens, int experts, int top_k,
                                    int hidden, const PeerDispatch& peer, int sms,
                                    cudaStream_t stream) {
  if (tokens <= 0) return cudaSuccess;
  if (peer.x_base == nullptr || peer.ret_base == nullptr || peer.dest_off == nullptr ||
      peer.local < 1 || top_k < 1 || top_k > 8 || sms < 2) {
    return cudaErrorInvalidValue;
  }
  const bool vec = hidden % 4 == 0 && aligned_to(x, 16);
  const void* fn = vec ? reinterpret_cast<const void*>(ep_dispatch_rest_kernel<true>)
                       : reinterpret_cast<const void*>(ep_dispatch_rest_kernel<false>);
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       kRestSmem);
  if (e != cudaSuccess) return e;
  // Clusters of two CTAs: the SMs taken come in pairs inside a GPC, so every
  // GPC keeps an even number of free SMs for the GEMM's CTA pairs.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(sms & ~1));
  cfg.blockDim = dim3(kRestThreads);
  cfg.dynamicSmemBytes = kRestSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = vec ? cudaLaunchKernelEx(&cfg, ep_dispatch_rest_kernel<true>, x, ids, offsets, route_pos,
                               tokens, experts, top_k, hidden, peer)
          : cudaLaunchKernelEx(&cfg, ep_dispatch_rest_kernel<false>, x, ids, offsets, route_pos,
                               tokens, experts, top_k, hidden, peer);
  if (e != cudaSuccess) return e;
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_token_permute_cursor(const float* x, const int32_t* ids,
                                        const int32_t* offsets, int32_t* cursors,
                                        float* x_permuted, int32_t* route_pos,
                                        int32_t* sorted_route, int tokens, int top_k, int hidden,
                                        cudaStream_t stream) {
  if (tokens <= 0) return cudaSuccess;
  const int routes = tokens * top_k;
  permute_cursor_rank_kernel<<<1, 1024, 0, stream>>>(ids, offsets, cursors, route_pos,
                                                     sorted_route, routes);
  note_launch();
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess || hidden <= 0) return err;
  const bool vec = hidden % 4 == 0 && aligned_to(x, 16) && aligned_to(x_permuted, 16);
  const int blocks = min(ceil_div(tokens, 8), 8 * sm_count());
  if (vec) {
    permute_copy_kernel<true><<<blocks, 256, 0, stream>>>(x, route_pos, x_permuted, tokens, top_k,
                                                          hidden);
  } else {
    permute_copy_kernel<false><<<blocks, 256, 0, stream>>>(x, route_pos, x_permuted, tokens,
                                                           top_k, hidden);
  }
  note_launch();
  return cudaGetLastError();
}

}  // namespace rrb
