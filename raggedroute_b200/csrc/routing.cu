// Routing metadata for B200: histogram, exclusive scan and the fused
// histogram + exclusive scan.
//
// Semantics follow the reference: counts[e] = #{r : ids[r] == e} with ids
// outside [0, E) skipped (src/histogram/cuda_naive/baseline.cu:17-27);
// offsets[0] = 0, offsets[e+1] = offsets[e] + counts[e], alias-safe
// (src/scan/cuda_naive/baseline.cu:12-26). Integer results are exact and
// independent of scheduling.
//
// Design: ids stream through 128-bit loads; each CTA keeps R shared-memory
// copies of its histogram (R a power of two, 32 for E <= 256, fewer for more
// experts so that the copies fit in 40 KB) and lane l adds to copy l % R with
// a plain shared atomic. The copies are E + 1 words apart, so the same
// expert's counters in different copies sit in different banks: an
// all-to-one-expert input conflicts at most 32 / R ways per instruction and a
// spread-out input touches mostly distinct banks; the copies are folded at
// the end. (Warp aggregation
// with __match_any_sync, measured earlier, costs in proportion to the number
// of distinct experts in a warp: 1M uniform routes took 14.4 us over 256
// experts against 6.2 us over one.) Three ways to merge the CTA histograms,
// by size:
//   * up to 32K routes: one CTA does everything (no merge, no reset);
//   * up to 256K routes: one thread-block cluster (16 CTAs, or 8 where a
//     16-CTA cluster cannot be placed); after a cluster barrier CTA 0 sums
//     the CTAs' histograms through distributed shared memory and writes
//     counts (and the scan) directly, so there is no reset launch and no
//     global atomic, and a second barrier keeps every CTA's shared memory
//     alive until CTA 0 has read it;
//   * beyond: CTAs merge into zeroed counts with one global atomic per
//     non-empty bin, and the fused operator then scans in a second, one-CTA
//     launch (measured at 1M routes: a last-CTA scan behind a ticket and a
//     fence inside the same launch was slower than the separate scan).
#include <cooperative_groups.h>

#include <mutex>

#include "common.cuh"

namespace rrb {
namespace {

constexpr int kHistThreads = 512;
// Up to this many routes the fused operator runs in a single CTA.
constexpr int kFusedSingleCtaMaxRoutes = 1 << 15;
// Shared memory for a CTA's histogram copies: copy r of counter e is
// hist[r * (E + 1) + e].
constexpr int kReplicaBytes = 40 * 1024;

// Copies for E experts: the largest power of two <= 32 that fits.
int hist_replicas(int experts) {
  int r = 32;
  while (r > 1 && static_cast<long long>(r) * (experts + 1) * 4 > kReplicaBytes) r >>= 1;
  return r;
}

std::size_t hist_smem(int experts) {
  return static_cast<std::size_t>(hist_replicas(experts)) * (experts + 1) * sizeof(int);
}

__device__ __forceinline__ void warp_add(int* mine, int e, int experts) {
  if (e >= 0 && e < experts) atomicAdd(mine + e, 1);
}

// Zeroes the copies. All threads of the CTA; a barrier must follow.
__device__ __forceinline__ void zero_replicas(int* hist, int experts, int reps) {
  for (int i = threadIdx.x; i < reps * (experts + 1); i += blockDim.x) hist[i] = 0;
}

// Folds the copies into hist[0..experts). All threads; call after a barrier
// that follows the accumulation; a barrier must follow.
__device__ __forceinline__ void fold_replicas(int* hist, int experts, int reps) {
  for (int i = threadIdx.x; i < experts; i += blockDim.x) {
    int v = hist[i];
    for (int r = 1; r < reps; ++r) v += hist[r * (experts + 1) + i];
    hist[i] = v;
  }
}

// Adds the histogram of ids[begin, end) (a contiguous slice per CTA) to the
// shared histogram copies. All threads of the CTA must call it.
__device__ void accumulate_slice(const int32_t* __restrict__ ids, long long begin, long long end,
                                 int* hist, int experts, int reps, bool vec) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int warps = blockDim.x >> 5;
  int* mine = hist + (lane & (reps - 1)) * (experts + 1);
  if (vec) {
    // begin is a multiple of 4 and ids is 16-byte aligned.
    const long long n4 = (end - begin) >> 2;
    const int4* src = reinterpret_cast<const int4*>(ids + begin);
    constexpr int kUnroll = 4;  // 4 x 128-bit loads in flight per lane
    for (long long base = static_cast<long long>(warp) * 32 * kUnroll; base < n4;
         base += static_cast<long long>(warps) * 32 * kUnroll) {
      int4 v[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const long long i = base + u * 32 + lane;
        v[u] = i < n4 ? __ldg(src + i) : make_int4(-1, -1, -1, -1);
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        warp_add(mine, v[u].x, experts);
        warp_add(mine, v[u].y, experts);
        warp_add(mine, v[u].z, experts);
        warp_add(mine, v[u].w, experts);
      }
    }
    for (long long base = begin + (n4 << 2) + static_cast<long long>(warp) * 32; base < end;
         base += static_cast<long long>(warps) * 32) {
      const int e = (base + lane < end) ? __ldg(ids + base + lane) : -1;
      warp_add(mine, e, experts);
    }
  } else {
    for (long long base = begin + static_cast<long long>(warp) * 32; base < end;
         base += static_cast<long long>(warps) * 32) {
      const int e = (base + lane < end) ? __ldg(ids + base + lane) : -1;
      warp_add(mine, e, experts);
    }
  }
}

__device__ __forceinline__ void slice_of(long long routes, long long& begin, long long& end) {
  // Slices are multiples of 4 routes so vector loads stay aligned.
  const long long per = ((routes + gridDim.x - 1) / gridDim.x + 3) & ~3LL;
  begin = per * blockIdx.x;
  end = begin + per;
  if (begin > routes) begin = routes;
  if (end > routes) end = routes;
}

__global__ void __launch_bounds__(kHistThreads) histogram_accumulate_kernel(
    const int32_t* __restrict__ ids, int32_t* __restrict__ counts, int routes, int experts,
    int reps, bool vec) {
  extern __shared__ int hist[];
  zero_replicas(hist, experts, reps);
  __syncthreads();
  long long begin, end;
  slice_of(routes, begin, end);
  accumulate_slice(ids, begin, end, hist, experts, reps, vec);
  __syncthreads();
  fold_replicas(hist, experts, reps);
  __syncthreads();
  for (int i = threadIdx.x; i < experts; i += blockDim.x) {
    const int c = hist[i];
    if (c != 0) atomicAdd(counts + i, c);
  }
}

// Block-wide exclusive scan of up to blockDim.x (<= 1024) values, one per
// thread. Returns the exclusive prefix; *total receives the sum.
__device__ int block_exclusive_scan(int value, int* warp_sums, int* total) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  int inclusive = value;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, inclusive, off);
    if (lane >= off) inclusive += n;
  }
  if (lane == 31) warp_sums[warp] = inclusive;
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    int s = lane < nw ? warp_sums[lane] : 0;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, s, off);
      if (lane >= off) s += n;
    }
    if (lane < nw) warp_sums[lane] = s;  // inclusive over warps
  }
  __syncthreads();
  const int warp_prefix = warp == 0 ? 0 : warp_sums[warp - 1];
  *total = warp_sums[(blockDim.x >> 5) - 1];
  return warp_prefix + inclusive - value;
}

// Scans counts[0..experts) (experts <= 1024) into offsets[0..experts]. Reads
// everything before writing anything, so counts may alias offsets.
__device__ void scan_counts_to_offsets(const int32_t* counts, int32_t* offsets, int experts,
                                       int* warp_sums, bool bypass_l1) {
  const int t = threadIdx.x;
  int v = 0;
  if (t < experts) v = bypass_l1 ? __ldcg(counts + t) : counts[t];
  int total = 0;
  const int excl = block_exclusive_scan(v, warp_sums, &total);
  __syncthreads();
  if (t < experts) offsets[t] = excl;
  if (t == 0) offsets[experts] = total;
}

__global__ void __launch_bounds__(1024) exclusive_scan_kernel(const int32_t* counts,
                                                              int32_t* offsets, int experts) {
  __shared__ int warp_sums[32];
  scan_counts_to_offsets(counts, offsets, experts, warp_sums, false);
}

__global__ void __launch_bounds__(1024) hist_scan_single_kernel(const int32_t* __restrict__ ids,
                                                                int32_t* __restrict__ counts,
                                                                int32_t* __restrict__ offsets,
                                                                int routes, int experts,
                                                                int reps, bool vec) {
  extern __shared__ int hist[];
  __shared__ int warp_sums[32];
  zero_replicas(hist, experts, reps);
  __syncthreads();
  accumulate_slice(ids, 0, routes, hist, experts, reps, vec);
  __syncthreads();
  fold_replicas(hist, experts, reps);
  __syncthreads();
  const int t = threadIdx.x;
  const int v = t < experts ? hist[t] : 0;
  int total = 0;
  const int excl = block_exclusive_scan(v, warp_sums, &total);
  if (t < experts) {
    counts[t] = v;
    offsets[t] = excl;
  }
  if (t == 0) offsets[experts] = total;
}

constexpr int kClusterThreads = 1024;
// Up to this many routes the cluster kernel is used. Its 16 CTAs then hold
// at most 16K ids each; the shared-memory updates of a CTA grow with its
// slice (measured on B200 at 1M uniform routes over 256 experts: 69 us in
// one cluster against 15 us over 128 CTAs), so larger inputs take the
// many-CTA kernel.
constexpr long long kClusterMaxRoutes = 1LL << 18;

// One cluster (the whole grid): counts = histogram of ids; with kScan also
// offsets = exclusive scan of counts. experts <= 1024 = blockDim.x.
template <bool kScan>
__global__ void __launch_bounds__(kClusterThreads) hist_cluster_kernel(
    const int32_t* __restrict__ ids, int32_t* __restrict__ counts, int32_t* __restrict__ offsets,
    int routes, int experts, int reps, bool vec) {
  namespace cg = cooperative_groups;
  extern __shared__ int hist[];
  __shared__ int warp_sums[32];
  cg::cluster_group cluster = cg::this_cluster();
  zero_replicas(hist, experts, reps);
  __syncthreads();
  long long begin, end;
  slice_of(routes, begin, end);
  accumulate_slice(ids, begin, end, hist, experts, reps, vec);
  __syncthreads();
  fold_replicas(hist, experts, reps);
  cluster.sync();  // every CTA's folded histogram is complete and visible
  if (cluster.block_rank() == 0) {
    const int e = threadIdx.x;
    const int nblocks = static_cast<int>(cluster.num_blocks());
    int v = 0;
    if (e < experts) {
      for (int b = 0; b < nblocks; ++b) v += cluster.map_shared_rank(hist, b)[e];
      counts[e] = v;
    }
    if constexpr (kScan) {
      int total = 0;
      const int excl = block_exclusive_scan(v, warp_sums, &total);
      if (e < experts) offsets[e] = excl;
      if (e == 0) offsets[experts] = total;
    }
  }
  cluster.sync();  // CTA 0 has read every CTA's shared memory
}

// Expert-parallel receive offsets: group q = p * local + le holds the rows
// that source rank p routed to this rank's local expert le, i.e.
// count_all[p * experts + rank * local + le]; offsets are their exclusive scan.
__global__ void __launch_bounds__(1024) ep_recv_offsets_kernel(const int32_t* __restrict__ count_all,
                                                               int32_t* __restrict__ recv_offsets,
                                                               int nranks, int experts, int rank,
                                                               int local) {
  __shared__ int warp_sums[32];
  const int groups = nranks * local;  // <= 1024
  const int q = threadIdx.x;
  int v = 0;
  if (q < groups) {
    const int p = q / local;
    const int le = q - p * local;
    v = count_all[static_cast<long long>(p) * experts + rank * local + le];
  }
  int total = 0;
  const int excl = block_exclusive_scan(v, warp_sums, &total);
  if (q < groups) recv_offsets[q] = excl;
  if (q == 0) recv_offsets[groups] = total;
}

// Peer-transport layout. Rank d's receive buffer holds its local experts in
// order and, inside an expert, the rows of source ranks 0..G-1 in order, so
// its grouped GEMM sees plain contiguous expert segments. One CTA, one
// thread per (virtual) expert.
__global__ void __launch_bounds__(1024) ep_peer_layout_kernel(
    const int32_t* __restrict__ count_all, int32_t* __restrict__ dest_off,
    int32_t* __restrict__ recv_offsets, int nranks, int experts, int rank, int local,
    long long capacity, unsigned* err) {
  __shared__ long long column[kMaxExperts];  // rows of expert v over all sources
  const int v = threadIdx.x;
  long long col = 0, before = 0;
  if (v < experts) {
    for (int s = 0; s < nranks; ++s) {
      const int c = count_all[static_cast<long long>(s) * experts + v];
      if (s < rank) before += c;
      col += c;
    }
    column[v] = col;
  }
  __syncthreads();
  if (v >= experts) return;
  const int owner = v / local;
  const int le = v - owner * local;
  long long base = 0;
  for (int j = owner * local; j < v; ++j) base += column[j];
  const long long off = base + before;
  dest_off[v] = static_cast<int32_t>(off < capacity ? off : capacity);
  if (owner == rank) {
    recv_offsets[le] = static_cast<int32_t>(base < capacity ? base : capacity);
    if (le == local - 1) {
      const long long end = base + col;
      if (end > capacity) raise_device_error(err, kErrEpCapacity);
      recv_offsets[local] = static_cast<int32_t>(end < capacity ? end : capacity);
    }
  }
}

// CTAs per cluster for hist_cluster_kernel: 16 (non-portable) when the GPU
// can place such a cluster of 1024-thread CTAs, else 8. Queried once.
int hist_cluster_size() {
  static std::once_flag once;
  static int size = 8;
  std::call_once(once, [] {
    const void* fns[2] = {reinterpret_cast<const void*>(hist_cluster_kernel<false>),
                          reinterpret_cast<const void*>(hist_cluster_kernel<true>)};
    bool ok = true;
    for (const void* f : fns) {
      ok = ok && cudaFuncSetAttribute(f, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) ==
                     cudaSuccess;
    }
    if (ok) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(16);
      cfg.blockDim = dim3(kClusterThreads);
      cfg.dynamicSmemBytes = kReplicaBytes;  // the most any launch asks for
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = 16;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      int clusters = 0;
      for (const void* f : fns) {
        ok = ok && cudaOccupancyMaxActiveClusters(&clusters, f, &cfg) == cudaSuccess &&
             clusters > 0;
      }
    }
    if (ok) size = 16;
    cudaGetLastError();
  });
  return size;
}

template <bool kScan>
cudaError_t launch_hist_cluster(const int32_t* ids, int32_t* counts, int32_t* offsets, int routes,
                                int experts, bool vec, cudaStream_t stream) {
  const int size = hist_cluster_size();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(size);
  cfg.blockDim = dim3(kClusterThreads);
  cfg.dynamicSmemBytes = hist_smem(experts);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = size;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t err =
      cudaLaunchKernelEx(&cfg, hist_cluster_kernel<kScan>, ids, counts, offsets, routes, experts,
                         hist_replicas(experts), vec);
  if (err != cudaSuccess) return err;
  note_launch();
  return cudaGetLastError();
}

// A cluster launch the device cannot place (an MPS or MIG share with fewer
// SMs per GPC, for instance) is refused at launch time without touching the
// stream; the caller then takes the many-CTA path instead.
bool cluster_launch_refused(cudaError_t e) {
  return e == cudaErrorInvalidClusterSize || e == cudaErrorLaunchOutOfResources ||
         e == cudaErrorNotSupported || e == cudaErrorInvalidConfiguration;
}

int hist_grid(long long routes) {
  const int want = ceil_div(routes, kHistThreads * 16LL);
  const int cap = 2 * sm_count();
  return want < 1 ? 1 : (want > cap ? cap : want);
}

}  // namespace

cudaError_t launch_histogram_accumulate(const int32_t* ids, int32_t* counts, int routes,
                                        int experts, cudaStream_t stream) {
  if (routes <= 0) return cudaSuccess;
  const bool vec = aligned_to(ids, 16);
  histogram_accumulate_kernel<<<hist_grid(routes), kHistThreads, hist_smem(experts), stream>>>(
      ids, counts, routes, experts, hist_replicas(experts), vec);
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_histogram(const int32_t* ids, int32_t* counts, int routes, int experts,
                             cudaStream_t stream) {
  if (routes > kFusedSingleCtaMaxRoutes && routes <= kClusterMaxRoutes) {
    const cudaError_t e = launch_hist_cluster<false>(ids, counts, nullptr, routes, experts,
                                                     aligned_to(ids, 16), stream);
    if (!cluster_launch_refused(e)) return e;
    cudaGetLastError();
  }
  cudaError_t err = cudaMemsetAsync(counts, 0, sizeof(int32_t) * experts, stream);
  if (err != cudaSuccess) return err;
  return launch_histogram_accumulate(ids, counts, routes, experts, stream);
}

cudaError_t launch_exclusive_scan(const int32_t* counts, int32_t* offsets, int experts,
                                  cudaStream_t stream) {
  const int threads = ((experts + 31) / 32) * 32;
  exclusive_scan_kernel<<<1, threads < 32 ? 32 : threads, 0, stream>>>(counts, offsets, experts);
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_histogram_exclusive_scan(const int32_t* ids, int32_t* counts,
                                            int32_t* offsets, int routes, int experts,
                                            cudaStream_t stream) {
  const bool vec = aligned_to(ids, 16);
  if (routes <= kFusedSingleCtaMaxRoutes) {
    hist_scan_single_kernel<<<1, 1024, hist_smem(experts), stream>>>(
        ids, counts, offsets, routes, experts, hist_replicas(experts), vec);
    note_launch();
    return cudaGetLastError();
  }
  if (routes <= kClusterMaxRoutes) {
    const cudaError_t e =
        launch_hist_cluster<true>(ids, counts, offsets, routes, experts, vec, stream);
    if (!cluster_launch_refused(e)) return e;
    cudaGetLastError();
  }
  cudaError_t err = cudaMemsetAsync(counts, 0, sizeof(int32_t) * experts, stream);
  if (err != cudaSuccess) return err;
  err = launch_histogram_accumulate(ids, counts, routes, experts, stream);
  if (err != cudaSuccess) return err;
  return launch_exclusive_scan(counts, offsets, experts, stream);
}

cudaError_t launch_ep_recv_offsets(const int32_t* count_all, int32_t* recv_offsets, int nranks,
                                   int experts, int rank, int local, cudaStream_t stream) {
  ep_recv_offsets_kernel<<<1, 1024, 0, stream>>>(count_all, recv_offsets, nranks, experts, rank,
                                                 local);
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_ep_peer_layout(const int32_t* count_all, int32_t* dest_off,
                                  int32_t* recv_offsets, int nranks, int experts, int rank,
                                  int local, long long capacity, unsigned* err,
                                  cudaStream_t stream) {
  if (experts > kMaxExperts || local < 1) return cudaErrorInvalidValue;
  ep_peer_layout_kernel<<<1, 1024, 0, stream>>>(count_all, dest_off, recv_offsets, nranks,
                                                experts, rank, local, capacity, err);
  note_launch();
  return cudaGetLastError();
}

}  // namespace rrb
