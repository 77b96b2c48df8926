// Device-side tile schedule for the ragged grouped GEMM.
//
// The host never reads offsets (the reference chain passes R as a worst-case
// launch bound, src/grouped_gemm/operator.cpp:17-49), so every CTA of a
// persistent grid derives the schedule itself: expert e owns
// ceil(count_e / BM) * ceil(N / BN) output tiles, and a shared-memory
// exclusive prefix of those counts maps a linear tile index to
// (expert, m-tile, n-tile) by binary search. Empty experts own no tiles and
// ragged tails are a partial last m-tile. offsets == nullptr describes one
// group of `rows` rows (the dense GEMM).
#pragma once

#include "common.cuh"

namespace rrb {

struct TileCoord {
  int expert;
  int row0;     // first global row of the tile
  int row_end;  // end of the expert's segment (exclusive)
  int col0;
};

// prefix has experts + 1 entries. Call with all threads of the CTA; returns
// the total tile count. scratch needs 33 ints.
__device__ __forceinline__ int build_tile_prefix(const int32_t* __restrict__ offsets, int experts,
                                                 int rows, int bm, int n_tiles_n, int* prefix,
                                                 int* scratch) {
  if (offsets == nullptr) {
    if (threadIdx.x == 0) {
      prefix[0] = 0;
      prefix[1] = ((rows + bm - 1) / bm) * n_tiles_n;
    }
    __syncthreads();
    return prefix[1];
  }
  // Each thread sums a contiguous run of experts, then a block scan.
  const int nt = blockDim.x;
  const int per = (experts + nt - 1) / nt;
  const int e0 = threadIdx.x * per;
  const int e1 = min(experts, e0 + per);
  int local = 0;
  for (int e = e0; e < e1; ++e) {
    const int cnt = __ldg(offsets + e + 1) - __ldg(offsets + e);
    local += cnt > 0 ? ((cnt + bm - 1) / bm) * n_tiles_n : 0;
  }
  // Block exclusive scan of `local`.
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  int incl = local;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += v;
  }
  if (lane == 31) scratch[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int nw = nt >> 5;
    int s = lane < nw ? scratch[lane] : 0;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, s, off);
      if (lane >= off) s += v;
    }
    if (lane < nw) scratch[lane] = s;
  }
  __syncthreads();
  int run = (warp == 0 ? 0 : scratch[warp - 1]) + incl - local;
  for (int e = e0; e < e1; ++e) {
    prefix[e] = run;
    const int cnt = __ldg(offsets + e + 1) - __ldg(offsets + e);
    run += cnt > 0 ? ((cnt + bm - 1) / bm) * n_tiles_n : 0;
  }
  if (threadIdx.x == nt - 1) prefix[experts] = run;
  __syncthreads();
  return prefix[experts];
}

__device__ __forceinline__ TileCoord tile_coord(int t, const int32_t* __restrict__ offsets,
                                                int experts, int rows, const int* prefix, int bm,
                                                int bn, int n_tiles_n) {
  int e = 0;
  if (offsets != nullptr) {
    // Largest e with prefix[e] <= t (and a non-empty tile range).
    int lo = 0, hi = experts - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (prefix[mid] <= t) lo = mid; else hi = mid - 1;
    }
    e = lo;
  }
  const int local = t - prefix[e];
  const int mt = local / n_tiles_n;
  // The n-tiles of one row block are visited in an order rotated by the
  // block's global index t / n_tiles_n (prefix[e] is a multiple of
  // n_tiles_n, so this permutes tiles within a row block only). A persistent
  // CTA that takes every units-th tile would otherwise see only the n-tiles
  // congruent to its own index modulo gcd(units, n_tiles_n): with 74 CTA
  // pairs and 6 n-tiles (N = 1408), the narrower last n-tile would fall to
  // the odd pairs only, and the even pairs would carry ~10% more work.
  const int ntile = (local - mt * n_tiles_n + t / n_tiles_n) % n_tiles_n;
  TileCoord c;
  c.expert = e;
  const int base = offsets != nullptr ? __ldg(offsets + e) : 0;
  c.row0 = base + mt * bm;
  c.row_end = offsets != nullptr ? __ldg(offsets + e + 1) : rows;
  c.col0 = ntile * bn;
  return c;
}

}  // namespace rrb
