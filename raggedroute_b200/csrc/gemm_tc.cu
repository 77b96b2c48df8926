// Ragged grouped GEMM on the 5th-generation tensor cores (tcgen05, sm_100a)
// with a 3xTF32 split that holds an FP32-accuracy contract.
//
// Contract (src/grouped_gemm/cuda_naive/baseline.cu:11-31 of the reference):
// y[r, :] = x[r, :] . W[e] for r in [offsets[e], offsets[e+1]); rows outside
// every segment are untouched. The dense router GEMM is the same kernel with
// one implicit group.
//
// 3xTF32: every operand element v is split into hi = rna_tf32(v) and
// lo = rna_tf32(v - hi) (v - hi is exact in FP32). Per k-step the tensor core
// accumulates lo_a*hi_b + hi_a*lo_b + hi_a*hi_b into an FP32 TMEM
// accumulator; the dropped lo_a*lo_b term and the TF32 rounding of lo are
// below 2^-21 relative per product. The tensor core's own accumulate step
// loses precision with a consistent bias (measured: 2.9e-5 normwise at
// K=4096), so the accumulator is promoted every 512 of K: each chunk is
// accumulated from zero into the partial P (TMEM columns 0-255) and added,
// with round-to-nearest FP32 adds on the CUDA cores, into the running sum S
// (TMEM columns 256-511). The last chunk's S + P goes straight to global.
//
// Structure: a persistent CTA per SM walks the device-side tile schedule
// (tile_sched.cuh, read from offsets, no host sync). Tiles are 128 rows x 256
// columns; warps are specialised:
//   warp 0     TMA producer: A (x rows, K-major, 64-byte swizzle) and B (the
//              expert's [K, N] weights, N-major, 128-byte swizzle) per 16-wide
//              k-block into a 4-slot raw ring; no multicast.
//   warp 1     MMA issuer: 3 tcgen05.mma (M=128, N<=256, K=8) per k-step into
//              P; it waits for P to be promoted before the next chunk.
//   warps 2-17 workers (16 warps = 4 TMEM lane quarters x 4 column groups):
//              (a) split: hi/lo of each landed k-block into a 2-slot operand
//              ring. kind::tf32 MMAs take K-major operands only (an N-major B
//              reads as zeros on sm_100a), so B is transposed to K-major here
//              with a bank-conflict-free lane mapping; the raw slot is released
//              as soon as it has been read.
//              (b) promotion: S = P, S += P, or y = S + P for the tile's last
//              chunk, each thread covering 64 columns of one TMEM lane.
//              Promotion of chunk c runs after the first k-block of the next
//              chunk has been split, so the MMA resumes at once.
// A partial last m-tile of an expert is loaded shifted back so it ends at the
// segment end: TMA never reads a row at or beyond offsets[E], and rows before
// the segment come from the previous expert (computed, never stored) or are
// zero-filled when negative. Every mbarrier wait is bounded (2 s); on a timeout
// the kernel records kErrMbarTimeout, drains its own TMA loads and MMAs,
// frees its TMEM and returns.
#include <cuda.h>

#include <cstdlib>
#include <mutex>

#include "sm100.cuh"
#include "tile_sched.cuh"

namespace rrb {
namespace {

using namespace sm100;

// kPair = 1: one CTA per 128 x 256 tile (cta_group::1).
// kPair = 2: a CTA pair per 256 x 256 tile (cta_group::2): each CTA loads and
// splits its own 128 rows of A and its half of the tile's B columns, the even
// CTA issues M=256 MMAs that read both CTAs' shared memory, and each CTA
// accumulates its 128 rows in its own TMEM. Per SM this halves the B tile
// that is loaded, split and read by the tensor core.
template <int kPair>
struct Cfg {
  static constexpr int kRowsCta = 128;              // A rows / TMEM lanes per CTA
  static constexpr int kTileM = kRowsCta * kPair;   // output rows per tile
  static constexpr int kTileN = 256;                // output columns per tile
  static constexpr int kBCols = kTileN / kPair;     // B columns held per CTA
  static constexpr int kBK = 16;                    // fp32 elements per k-block
  static constexpr int kRawStages = 4;              // TMA ring
  static constexpr int kOpStages = kPair == 1 ? 2 : 4;  // hi/lo operand ring
  static constexpr int kABytes = kRowsCta * kBK * 4;    // 8 KB (64 B rows)
  static constexpr int kBChunkBytes = 32 * kBK * 4;     // 2 KB: 32 columns x 16 k rows
  static constexpr int kBBytes = kBCols * kBK * 4;
  static constexpr int kRawBytes = kABytes + kBBytes;   // A raw | B raw (N-major)
  static constexpr int kOpBytes = 2 * (kABytes + kBBytes);  // A hi | A lo | B hi | B lo
  static constexpr int kOffBRaw = kABytes;
  static constexpr int kOffAHi = 0;
  static constexpr int kOffALo = kABytes;
  static constexpr int kOffBHi = 2 * kABytes;
  static constexpr int kOffBLo = 2 * kABytes + kBBytes;
};

constexpr int kChunkKb = 32;      // k-blocks per promoted chunk (K = 512)
constexpr uint32_t kColP = 0;     // TMEM columns of the chunk partial
constexpr uint32_t kColS = 256;   // TMEM columns of the running sum
constexpr int kWorkerWarps = 16;
constexpr int kFirstWorkerWarp = 2;
constexpr int kThreads = (kFirstWorkerWarp + kWorkerWarps) * 32;  // 576
constexpr int kTmemCols = 512;
constexpr int kWorkerThreads = kWorkerWarps * 32;
constexpr int kEpiCols = 256 / 4;  // columns per worker thread

template <int kPair>
struct alignas(1024) Smem {
  using C = Cfg<kPair>;
  uint8_t raw[C::kRawStages][C::kRawBytes];
  uint8_t op[C::kOpStages][C::kOpBytes];
  uint64_t raw_full[C::kRawStages];
  uint64_t raw_empty[C::kRawStages];
  uint64_t op_full[C::kOpStages];   // pairs: counted in the even CTA only
  uint64_t op_empty[C::kOpStages];
  uint64_t tmem_full;   // P holds a finished chunk
  uint64_t tmem_empty;  // P has been promoted (pairs: even CTA only)
  uint64_t mma_done;
  uint32_t tmem_base;
  int failed;
  int issued[C::kRawStages];
  int prefix[kMaxExperts + 1];
  int scratch[33];
};

template <int kPair>
constexpr std::size_t smem_bytes() {
  return sizeof(Smem<kPair>) + 1024;
}

struct TileGeom {
  int expert, row0, row_end, base, col0, ncols, n_mma;
};

template <int kPair>
__device__ __forceinline__ TileGeom geom(int t, const int32_t* offsets, int experts, int rows,
                                         const int* prefix, int n_tiles_n, int output) {
  using C = Cfg<kPair>;
  const TileCoord c = tile_coord(t, offsets, experts, rows, prefix, C::kTileM, C::kTileN,
                                 n_tiles_n);
  TileGeom g;
  g.expert = c.expert;
  g.row0 = c.row0;
  g.row_end = c.row_end;
  g.base = (c.row0 + C::kTileM > c.row_end) ? c.row_end - C::kTileM : c.row0;
  g.col0 = c.col0;
  g.ncols = min(C::kTileN, output - c.col0);
  // MMA N: a multiple of 16 per CTA's share of B.
  const int q = 16 * kPair;
  g.n_mma = (g.ncols + q - 1) / q * q;
  return g;
}

__device__ __forceinline__ void split4(const float4 v, float4& h, float4& l) {
  h.x = tf32_rna(v.x);
  h.y = tf32_rna(v.y);
  h.z = tf32_rna(v.z);
  h.w = tf32_rna(v.w);
  l.x = tf32_rna(v.x - h.x);
  l.y = tf32_rna(v.y - h.y);
  l.z = tf32_rna(v.z - h.z);
  l.w = tf32_rna(v.w - h.w);
}

// Byte offset of 16-byte chunk kc (k = 4*kc..4*kc+3) of row r in a K-major
// tile of 16 fp32 per row with the 64-byte swizzle (TMA and UMMA agree on it).
__device__ __forceinline__ int kmajor64_offset(int r, int kc) {
  return r * 64 + ((kc ^ ((r >> 1) & 3)) << 4);
}

// Element (k, n) of the N-major raw B tile: 32-column chunks of 16 rows x
// 128 bytes with the 128-byte swizzle.
__device__ __forceinline__ int nmajor128_offset(int k, int n) {
  return (n >> 5) * (32 * 16 * 4) + k * 128 + ((((n & 31) >> 2) ^ (k & 7)) << 4) +
         ((n & 3) << 2);
}

template <int kPair>
__global__ void __launch_bounds__(kThreads, 1) grouped_gemm_tc_kernel(
    const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
    const int32_t* __restrict__ offsets, float* __restrict__ y, int experts, int rows,
    int hidden, int output, int wsets, unsigned* err, const RowScatter scatter) {
  using C = Cfg<kPair>;
  extern __shared__ uint8_t smem_raw[];
  Smem<kPair>& s = *reinterpret_cast<Smem<kPair>*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_tiles_n = (output + C::kTileN - 1) / C::kTileN;
  const int num_kb = (hidden + C::kBK - 1) / C::kBK;
  const uint32_t rank = kPair == 1 ? 0u : cluster_ctarank();
  const bool leader = rank == 0;
  // Work unit: a CTA (kPair = 1) or a CTA pair (kPair = 2).
  const int unit = blockIdx.x / kPair;
  const int units = gridDim.x / kPair;

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::kRawStages; ++i) {
      mbar_init(&s.raw_full[i], 1);
      mbar_init(&s.raw_empty[i], kWorkerWarps);
      s.issued[i] = 0;
    }
    // In the even CTA of a pair, op_full and tmem_empty also count the one
    // forwarded arrival of the odd CTA's relay thread.
    const uint32_t counted = kWorkerWarps + (kPair == 2 && leader ? 1 : 0);
    for (int i = 0; i < C::kOpStages; ++i) {
      mbar_init(&s.op_full[i], counted);
      mbar_init(&s.op_empty[i], 1);
    }
    mbar_init(&s.tmem_full, 1);
    mbar_init(&s.tmem_empty, counted);
    mbar_init(&s.mma_done, 1);
    s.failed = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    if constexpr (kPair == 1) {
      tmem_alloc(&s.tmem_base, kTmemCols);
      tmem_relinquish();
    } else {
      tmem_alloc_pair(&s.tmem_base, kTmemCols);
      tmem_relinquish_pair();
    }
  }
  const int total =
      build_tile_prefix(offsets, experts, rows, C::kTileM, n_tiles_n, s.prefix, s.scratch);
  tc_fence_before();
  __syncthreads();
  if constexpr (kPair == 2) cluster_sync();  // the peer's barriers are initialised
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;
  volatile int* failed = &s.failed;
  // The MMA issuer's waits; in a pair they complete with an arrival from the
  // other CTA, so they acquire at cluster scope.
  auto wait_issuer = [&](uint64_t* bar, uint32_t parity) {
    if constexpr (kPair == 1) {
      return mbar_wait(bar, parity, err, failed);
    } else {
      return mbar_wait_cluster(bar, parity, err, failed);
    }
  };

  if (warp == 0) {
    // ---------------- TMA producer: this CTA's A rows and B columns ----------------
    if (lane == 0) {
      tma_prefetch_desc(&tma_a);
      tma_prefetch_desc(&tma_b);
      int stage = 0;
      uint32_t phase = 0;
      for (int t = unit; t < total && !*failed; t += units) {
        const TileGeom g = geom<kPair>(t, offsets, experts, rows, s.prefix, n_tiles_n, output);
        const int half = g.n_mma / kPair;
        const int bcol0 = g.col0 + static_cast<int>(rank) * half;
        const int nchunks = (half + 31) >> 5;
        const int arow0 = g.base + static_cast<int>(rank) * C::kRowsCta;
        const uint32_t bytes = C::kABytes + nchunks * C::kBChunkBytes;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&s.raw_empty[stage], phase ^ 1u, err, failed)) break;
          uint8_t* st = s.raw[stage];
          mbar_arrive_expect_tx(&s.raw_full[stage], bytes);
          tma_load_2d(st, &tma_a, &s.raw_full[stage], kb * C::kBK, arow0);
          for (int j = 0; j < nchunks; ++j) {
            tma_load_3d(st + C::kOffBRaw + j * C::kBChunkBytes, &tma_b, &s.raw_full[stage],
                        bcol0 + 32 * j, kb * C::kBK, g.expert % wsets);
          }
          s.issued[stage] += 1;
          if (++stage == C::kRawStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1 && kPair == 2 && !leader) {
    // ---------------- relay (odd CTA of a pair) ----------------
    // Forwards each completed phase of this CTA's op_full (operands split) and
    // tmem_empty (chunk promoted) to the even CTA's barrier, in the order the
    // workers produce them. One release at cluster scope per phase, by a
    // thread with no stores of its own in flight.
    if (lane == 0) {
      int ostage = 0;
      uint32_t ophase = 0, acc_phase = 0;
      bool pending = false;
      int t = unit;
      int kb = 0;
      while (!*failed) {
        const bool have_block = t < total;
        if (have_block) {
          if (!mbar_wait(&s.op_full[ostage], ophase, err, failed)) break;
          mbar_arrive_cluster(mapa_shared(smem_u32(&s.op_full[ostage]), 0));
          if (++ostage == C::kOpStages) {
            ostage = 0;
            ophase ^= 1u;
          }
        }
        if (pending) {
          if (!mbar_wait(&s.tmem_empty, acc_phase, err, failed)) break;
          mbar_arrive_cluster(mapa_shared(smem_u32(&s.tmem_empty), 0));
          acc_phase ^= 1u;
          pending = false;
        }
        if (!have_block) break;
        if ((kb + 1) % kChunkKb == 0 || kb + 1 == num_kb) pending = true;
        if (++kb == num_kb) {
          kb = 0;
          t += units;
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (the even CTA of a pair) ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = unit; t < total && ok && !*failed; t += units) {
        const TileGeom g = geom<kPair>(t, offsets, experts, rows, s.prefix, n_tiles_n, output);
        const uint32_t idesc = idesc_tf32(C::kTileM, g.n_mma, false, false);
        for (int kc = 0; kc < num_kb && ok; kc += kChunkKb) {
          if (!wait_issuer(&s.tmem_empty, acc_phase ^ 1u)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem + kColP;
          const int kend = min(num_kb, kc + kChunkKb);
          for (int kb = kc; kb < kend; ++kb) {
            if (!wait_issuer(&s.op_full[stage], phase)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t base = smem_u32(s.op[stage]);
            const uint32_t a_hi = base + C::kOffAHi;
            const uint32_t a_lo = base + C::kOffALo;
            const uint32_t b_hi = base + C::kOffBHi;
            const uint32_t b_lo = base + C::kOffBLo;
#pragma unroll
            for (int ks = 0; ks < C::kBK / 8; ++ks) {
              // K-major, 64-byte swizzle: 8-row groups 512 B apart; the second
              // k-step starts 32 B into each row.
              const uint64_t ah = smem_desc(a_hi + ks * 32, 16, 512, Swizzle::k64B);
              const uint64_t al = smem_desc(a_lo + ks * 32, 16, 512, Swizzle::k64B);
              const uint64_t bh = smem_desc(b_hi + ks * 32, 16, 512, Swizzle::k64B);
              const uint64_t bl = smem_desc(b_lo + ks * 32, 16, 512, Swizzle::k64B);
              const uint32_t first = (kb == kc && ks == 0) ? 0u : 1u;
              if constexpr (kPair == 1) {
                mma_tf32(d, al, bh, idesc, first);
                mma_tf32(d, ah, bl, idesc, 1u);
                mma_tf32(d, ah, bh, idesc, 1u);
              } else {
                mma_tf32_pair(d, al, bh, idesc, first);
                mma_tf32_pair(d, ah, bl, idesc, 1u);
                mma_tf32_pair(d, ah, bh, idesc, 1u);
              }
            }
            if constexpr (kPair == 1) {
              mma_commit(&s.op_empty[stage]);
            } else {
              mma_commit_pair(&s.op_empty[stage]);
            }
            if (++stage == C::kOpStages) {
              stage = 0;
              phase ^= 1u;
            }
          }
          if (!ok) break;
          if constexpr (kPair == 1) {
            mma_commit(&s.tmem_full);
          } else {
            mma_commit_pair(&s.tmem_full);
          }
          acc_phase ^= 1u;
        }
      }
      // All MMAs this thread issued are complete once mma_done fires.
      if constexpr (kPair == 1) {
        mma_commit(&s.mma_done);
      } else {
        mma_commit_pair(&s.mma_done);
      }
      int dummy = 0;
      mbar_wait(&s.mma_done, 0, err, &dummy);
    }
  } else {
    // ---------------- workers: split + promotion + store ----------------
    const int tid = threadIdx.x - kFirstWorkerWarp * 32;  // 0..511
    const int ew = warp - kFirstWorkerWarp;
    const int quarter = warp & 3;  // TMEM lanes this warp may access
    const int cgroup = ew >> 2;    // 64-column group of the tile
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    const bool vec = (output & 3) == 0;
    int rstage = 0, ostage = 0;
    uint32_t rphase = 0, ophase = 0, acc_phase = 0;
    // The chunk awaiting promotion (tile geometry + whether it ends its tile).
    bool pending = false, pending_first = false, pending_last = false;
    TileGeom pg{};
    int t = unit;
    int kb = 0;
    TileGeom g{};
    if (t < total) g = geom<kPair>(t, offsets, experts, rows, s.prefix, n_tiles_n, output);
    // This thread's B items (n, kc) of a k-block depend only on the tile's
    // column count, so their shared-memory offsets are computed once per
    // tile: item (n, kc) reads rows 4kc..4kc+3 of column n of the N-major raw
    // tile and writes 16 bytes of row n of the K-major operands. A warp
    // covers 32 consecutive n of one kc, so the scalar reads are
    // conflict-free and the 16-byte writes take the minimum 4 wavefronts.
    constexpr int kItems = (C::kBCols * 4 + kWorkerThreads - 1) / kWorkerThreads;
    uint32_t bsrc[kItems][4];
    uint32_t bdst[kItems];
    int b_items = 0;   // items of this thread in the current tile
    int b_for = -1;    // n_mma the offsets were computed for
    auto prepare_b = [&](int n_mma) {
      const int half = n_mma / kPair;
      const int nitems = (((half + 31) >> 5) << 5) * 4;
      b_items = 0;
#pragma unroll
      for (int i = 0; i < kItems; ++i) {
        const int it = tid + i * kWorkerThreads;
        if (it < nitems) b_items = i + 1;
        const int n = (it & 31) + ((it >> 7) << 5);
        const int kc = (it >> 5) & 3;
#pragma unroll
        for (int j = 0; j < 4; ++j) bsrc[i][j] = static_cast<uint32_t>(nmajor128_offset(4 * kc + j, n));
        bdst[i] = static_cast<uint32_t>(kmajor64_offset(n, kc));
      }
      b_for = n_mma;
    };
    // One iteration = split one k-block (while any remain), then promote the
    // previously finished chunk. A final iteration without a k-block drains
    // the last chunk.
    while (!*failed) {
      const bool have_block = t < total;
      if (have_block) {
        if (!mbar_wait(&s.raw_full[rstage], rphase, err, failed) ||
            !mbar_wait(&s.op_empty[ostage], ophase ^ 1u, err, failed)) {
          break;
        }
        const uint32_t raw = smem_u32(s.raw[rstage]);
        const uint32_t op = smem_u32(s.op[ostage]);
        // A: same K-major layout in and out (one 16-byte chunk per thread).
        {
          float4 h, l;
          split4(lds_v4(raw + tid * 16), h, l);
          sts_v4(op + C::kOffAHi + tid * 16, h);
          sts_v4(op + C::kOffALo + tid * 16, l);
        }
        // B: N-major raw -> K-major hi/lo.
        if (g.n_mma != b_for) prepare_b(g.n_mma);
        const uint32_t braw = raw + C::kOffBRaw;
        const uint32_t bhi = op + C::kOffBHi;
        const uint32_t blo = op + C::kOffBLo;
#pragma unroll
        for (int i = 0; i < kItems; ++i) {
          if (i < b_items) {
            float4 v;
            v.x = lds_f32(braw + bsrc[i][0]);
            v.y = lds_f32(braw + bsrc[i][1]);
            v.z = lds_f32(braw + bsrc[i][2]);
            v.w = lds_f32(braw + bsrc[i][3]);
            float4 h, l;
            split4(v, h, l);
            sts_v4(bhi + bdst[i], h);
            sts_v4(blo + bdst[i], l);
          }
        }
        // Order this thread's generic reads (raw) and writes (operands)
        // before the async proxy (next TMA into raw, MMA reads of op).
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&s.raw_empty[rstage]);
          mbar_arrive(&s.op_full[ostage]);
        }
        if (++rstage == C::kRawStages) {
          rstage = 0;
          rphase ^= 1u;
        }
        if (++ostage == C::kOpStages) {
          ostage = 0;
          ophase ^= 1u;
        }
      }
      if (pending) {
        // Promotion of the finished chunk in P.
        if (!mbar_wait(&s.tmem_full, acc_phase, err, failed)) break;
        tc_fence_after();
        const int c_begin = cgroup * kEpiCols;
        const bool active = c_begin < pg.ncols;  // warp-uniform
        const int row = pg.base + static_cast<int>(rank) * C::kRowsCta + quarter * 32 + lane;
        bool store_row = pending_last && active && row >= pg.row0 && row < pg.row_end;
        float* out = y + static_cast<long long>(row) * output + pg.col0 + c_begin;
        if (scatter.dst != nullptr && store_row) {
          float* dst_row = scatter_row(scatter, row, output);
          store_row = dst_row != nullptr;
          out = dst_row + pg.col0 + c_begin;
        }
        const int w = min(kEpiCols, pg.ncols - c_begin);
        if (active) {
#pragma unroll
          for (int c = 0; c < kEpiCols; c += 16) {
            const uint32_t col = static_cast<uint32_t>(c_begin + c);
            uint32_t p[16];
            tmem_ld_32x32b_x16(tmem + kColP + col + lane_addr, p);
            if (!pending_first) {
              uint32_t q[16];
              tmem_ld_32x32b_x16(tmem + kColS + col + lane_addr, q);
              tmem_ld_wait();
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                p[j] = __float_as_uint(__uint_as_float(q[j]) + __uint_as_float(p[j]));
              }
            } else {
              tmem_ld_wait();
            }
            if (!pending_last) {
              tmem_st_32x32b_x16(tmem + kColS + col + lane_addr, p);
            } else if (store_row) {
              if (vec) {
#pragma unroll
                for (int j = 0; j < 16; j += 4) {
                  if (c + j < w) {
                    *reinterpret_cast<float4*>(out + c + j) =
                        make_float4(__uint_as_float(p[j]), __uint_as_float(p[j + 1]),
                                    __uint_as_float(p[j + 2]), __uint_as_float(p[j + 3]));
                  }
                }
              } else {
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                  if (c + j < w) out[c + j] = __uint_as_float(p[j]);
                }
              }
            }
          }
          if (!pending_last) tmem_st_wait();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.tmem_empty);
        acc_phase ^= 1u;
        pending = false;
      }
      if (!have_block) break;
      // The k-block just split ends a chunk: it is promoted next iteration.
      if ((kb + 1) % kChunkKb == 0 || kb + 1 == num_kb) {
        pending = true;
        pending_first = kb < kChunkKb;
        pending_last = (kb + 1 == num_kb);
        pg = g;
      }
      if (++kb == num_kb) {
        kb = 0;
        t += units;
        if (t < total) g = geom<kPair>(t, offsets, experts, rows, s.prefix, n_tiles_n, output);
      }
    }
  }

  // Scattered rows may live in another rank's memory: complete those stores
  // before the kernel ends (the barrier that follows publishes them).
  if (scatter.dst != nullptr && warp >= kFirstWorkerWarp) __threadfence_system();
  __syncthreads();
  if (warp == 0 && lane == 0 && *failed) {
    // Drain TMA loads still in flight into this CTA's shared memory.
    for (int i = 0; i < C::kRawStages; ++i) {
      if (s.issued[i] > 0) {
        int dummy = 0;
        mbar_wait(&s.raw_full[i], static_cast<uint32_t>((s.issued[i] - 1) & 1), err, &dummy);
      }
    }
  }
  __syncthreads();
  // A pair stays resident until the even CTA's MMAs, which read the odd
  // CTA's shared memory, are complete (the issuer waited for mma_done).
  if constexpr (kPair == 2) cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    if constexpr (kPair == 1) {
      tmem_dealloc(tmem, kTmemCols);
    } else {
      tmem_dealloc_pair(tmem, kTmemCols);
    }
  }
}

// ---- host side ---------------------------------------------------------------------

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static std::once_flag once;
  static EncodeTiledFn fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiledFn>(p);
    } else {
      cudaGetLastError();
    }
  });
  return fn;
}

template <int kPair>
bool kernel_configured() {
  static std::once_flag once;
  static bool ok = false;
  std::call_once(once, [] {
    ok = cudaFuncSetAttribute(grouped_gemm_tc_kernel<kPair>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(smem_bytes<kPair>())) == cudaSuccess;
    if (!ok) cudaGetLastError();
  });
  return ok;
}

// CTA pairs that can be resident at once when RAGGEDROUTE_B200_GEMM_PAIRS=1
// (read at every launch); 0 otherwise. Measured at C5 shapes, pairs run at
// the same speed per computed row as single CTAs but their 256-row tiles pad
// ragged experts twice as much, so single CTAs are the default.
int pair_units() {
  static std::once_flag once;
  static int units = 0;
  std::call_once(once, [] {
    if (!kernel_configured<2>()) return;
    cudaLaunchConfig_t cfg{};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(2 * sm_count(), 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = smem_bytes<2>();
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, grouped_gemm_tc_kernel<2>, &cfg) != cudaSuccess) {
      cudaGetLastError();
      n = 0;
    }
    units = n;
  });
  const char* v = std::getenv("RAGGEDROUTE_B200_GEMM_PAIRS");
  if (v == nullptr || v[0] != '1') return 0;
  return units;
}

}  // namespace

bool tc_gemm_supported(const float* x, const float* w, const float* y, int hidden, int output) {
  if (hidden <= 0 || output <= 0) return false;
  if (hidden % 4 != 0 || output % 4 != 0) return false;  // 16-byte TMA row strides
  if (!aligned_to(x, 16) || !aligned_to(w, 16) || !aligned_to(y, 16)) return false;
  static const bool disabled = [] {
    const char* v = std::getenv("RAGGEDROUTE_B200_DISABLE_TCGEN05");
    return v != nullptr && v[0] == '1';
  }();
  return !disabled && encode_fn() != nullptr;
}

int grouped_gemm_tc_pairs() { return pair_units(); }

cudaError_t launch_grouped_gemm_tc(const float* x, const float* w, const int32_t* offsets,
                                   float* y, int experts, int rows, int hidden, int output,
                                   cudaStream_t stream, int weight_sets,
                                   const RowScatter* scatter) {
  const int wsets = weight_sets > 0 ? weight_sets : experts;
  EncodeTiledFn encode = encode_fn();
  if (encode == nullptr) return cudaErrorNotSupported;
  const int pairs = pair_units();
  const int pair = pairs > 0 ? 2 : 1;
  if (pair == 1 && !kernel_configured<1>()) return cudaErrorNotSupported;
  // A: x [rows, hidden] row-major, 128-row boxes (one CTA's rows). Shifted
  // last tiles never read at or past the last segment end, so the row extent
  // only has to cover it.
  const long long a_rows = rows > 0 ? rows : (1LL << 31) - 1;
  CUtensorMap ma{}, mb{};
  {
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(hidden), static_cast<cuuint64_t>(a_rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(hidden) * 4};
    const cuuint32_t box[2] = {16, 128};
    const cuuint32_t elem[2] = {1, 1};
    if (encode(&ma, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(x), dims, strides, box,
               elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
      return cudaErrorInvalidValue;
    }
  }
  {
    // B: W [experts, hidden, output] viewed as {output, hidden, experts}.
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(output), static_cast<cuuint64_t>(hidden),
                                static_cast<cuuint64_t>(wsets)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(output) * 4,
                                   static_cast<cuuint64_t>(output) * hidden * 4};
    const cuuint32_t box[3] = {32, 16, 1};
    const cuuint32_t elem[3] = {1, 1, 1};
    if (encode(&mb, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(w), dims, strides, box,
               elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
      return cudaErrorInvalidValue;
    }
  }
  const RowScatter sc = scatter != nullptr ? *scatter : RowScatter{};
  unsigned* err = device_error_word();
  const int tile_m = 128 * pair;
  int units = pair == 2 ? pairs : sm_count();
  if (offsets == nullptr) {
    const long long tiles = static_cast<long long>((rows + tile_m - 1) / tile_m) *
                            ((output + 255) / 256);
    if (tiles <= 0) return cudaSuccess;
    if (tiles < units) units = static_cast<int>(tiles);
  }
  if (pair == 1) {
    grouped_gemm_tc_kernel<1><<<units, kThreads, smem_bytes<1>(), stream>>>(
        ma, mb, offsets, y, experts, rows, hidden, output, wsets, err, sc);
  } else {
    cudaLaunchConfig_t cfg{};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(2 * units, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = smem_bytes<2>();
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, grouped_gemm_tc_kernel<2>, ma, mb, offsets, y,
                                             experts, rows, hidden, output, wsets, err, sc);
    if (e != cudaSuccess) return e;
  }
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_grouped_gemm(const float* x, const float* w, const int32_t* offsets, float* y,
                                int experts, int rows, int hidden, int output,
                                cudaStream_t stream, int weight_sets, const RowScatter* scatter) {
  if (tc_gemm_supported(x, w, y, hidden, output)) {
    return launch_grouped_gemm_tc(x, w, offsets, y, experts, rows, hidden, output, stream,
                                  weight_sets, scatter);
  }
  return launch_grouped_gemm_simt(x, w, offsets, y, experts, rows, hidden, output, stream,
                                  weight_sets, scatter);
}

}  // namespace rrb
