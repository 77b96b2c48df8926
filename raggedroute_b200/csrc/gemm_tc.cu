// Ragged grouped GEMM on the 5th-generation tensor cores (tcgen05, sm_100a)
// with a 3xTF32 split that holds an FP32-accuracy contract.
//
// Contract (src/grouped_gemm/cuda_naive/baseline.cu:11-31 of the reference):
// y[r, :] = x[r, :] . W[e] for r in [offsets[e], offsets[e+1]); rows outside
// every segment are untouched. The dense router GEMM is the same kernel with
// one implicit group.
//
// 3xTF32: every operand element v is split into hi and lo = v - hi (exact in
// FP32) and per k-step the tensor core accumulates lo_a*hi_b + hi_a*lo_b +
// hi_a*hi_b into an FP32 TMEM accumulator. B (the weights): hi =
// rna_tf32(v), lo = rna_tf32(v - hi). A (the tokens): hi = v with its low
// 13 mantissa bits dropped, which is exactly what a kind::tf32 MMA reads
// from raw FP32 bits, so the MMA takes A hi straight from the TMA'd raw tile
// and only A lo is written (the MMA keeps the top 11 of its up to 13
// significant bits). The dropped lo_a*lo_b term and the TF32 truncation or
// rounding of lo stay below 2^-20 relative per product (measured at C5:
// 3.73e-6 normwise against FP64, 3.60e-6 with a rounded A hi). The tensor
// core's own accumulate step loses precision with a consistent bias
// (measured: 2.9e-5 normwise at K=4096), so the accumulator is promoted every
// 512 of K: each chunk is accumulated from zero into the partial P (TMEM
// columns 0-255) and added, with round-to-nearest FP32 adds on the CUDA
// cores, into the running sum S (TMEM columns 256-511). The last chunk's
// S + P goes straight to global. rna_tf32 is done on the bit pattern with
// integer adds (sm100.cuh, tf32_rna): the conversion instruction issues at a
// fraction of the integer rate and the split is on the critical path.
//
// Measured at C5 (T=65536, K=4096, E=128, N=1408) on one B200, per launch
// (diagnostic builds of this kernel): the MMAs with TMA loads but no split
// work 6.1 ms; the split with TMA loads but no MMAs 7.7 ms; the TMA loads
// and barrier hand-offs alone 3.7 ms; everything 8.1 ms.
//
// Structure: a persistent CTA per SM walks the device-side tile schedule
// (tile_sched.cuh, read from offsets, no host sync). Tiles are 128 rows x 256
// columns, or, for one group with N <= 128 (the router GEMM), two 128-row
// m-tiles sharing a 128-column B tile with one accumulator each (kMT = 2;
// same shared-memory and TMEM footprint). Options that are separate
// instantiations, so the default kernel carries none of them: row gather
// (kGather, A rows fetched from x through a row map by the producer warp
// with cp.async) and, at run time, an output-row scatter to other ranks'
// memory (expert-parallel combine, skipped once the abort fence is set) or
// the unpermute fused into the epilogue (each row weighted and added into
// its token's row with global float reductions; RowScatter combine mode).
// Warps are specialised:
//   warp 0     TMA producer: A (x rows, K-major, 64-byte swizzle) and B (the
//              expert's [K, N] weights, N-major, unswizzled) per 16-wide
//              k-block into a 5-slot raw ring, one box each (measured: eight
//              2 KB B boxes per k-block instead of one cost 5% at C5); no
//              multicast.
//   warp 1     MMA issuer: 3 tcgen05.mma (M=128, N<=256, K=8) per k-step into
//              P, A hi from the raw slot, the rest from the operand slot; its
//              commit releases both slots. It waits for P to be promoted
//              before the next chunk.
//   warps 2-17 workers (16 warps = 4 TMEM lane quarters x 4 column groups):
//              (a) split: A lo and B hi/lo of each landed k-block into a
//              2-slot operand ring. kind::tf32 MMAs take K-major operands
//              only here (an N-major B read as zeros when tried), so B is
//              transposed to K-major with a bank-conflict-free lane mapping.
//              With row gathering the raw A tile is unswizzled, so A hi is
//              written to the operand slot too and the workers release the
//              raw slot as soon as they have read it.
//              (b) promotion: S += P, or y = S + P for the tile's last chunk
//              (a tile's first chunk is accumulated into S directly), each
//              thread covering 64 columns of one TMEM lane.
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

#include "gemm_split.cuh"
#include "sm100.cuh"
#include "tile_sched.cuh"

namespace rrb {
namespace {

using namespace sm100;

constexpr int kBM = 128;                           // output rows per tile = TMEM lanes
constexpr int kBN = 256;                           // output columns per tile
constexpr int kBK = 16;                            // fp32 elements per k-block
constexpr int kRawStages = 5;                      // TMA ring (5 vs 4: 8.90 -> 8.52 ms at C5)
constexpr int kOpStages = 2;                       // hi/lo operand ring
constexpr int kABytes = kBM * kBK * 4;             // 8 KB (64 B rows)
constexpr int kBBytes = kBN * kBK * 4;             // 16 KB
constexpr int kRawBytes = kABytes + kBBytes;       // 24 KB: A raw | B raw (N-major)
constexpr int kOpBytes = 2 * (kABytes + kBBytes);  // 48 KB: A hi | A lo | B hi | B lo
                                                   // (A hi only used when gathering)
constexpr int kChunkKb = 32;                       // k-blocks per promoted chunk (K = 512)
constexpr uint32_t kColP = 0;                      // TMEM columns of the chunk partial
constexpr uint32_t kColS = kBN;                    // TMEM columns of the running sum
constexpr int kWorkerWarps = 16;
constexpr int kFirstWorkerWarp = 2;
constexpr int kThreads = (kFirstWorkerWarp + kWorkerWarps) * 32;  // 576
constexpr int kTmemCols = 512;
constexpr int kWorkerThreads = kWorkerWarps * 32;
constexpr int kEpiCols = kBN / 4;                  // columns per worker thread

struct alignas(1024) Smem {
  uint8_t raw[kRawStages][kRawBytes];
  uint8_t op[kOpStages][kOpBytes];
  uint64_t raw_full[kRawStages];
  uint64_t raw_empty[kRawStages];
  uint64_t op_full[kOpStages];
  uint64_t op_empty[kOpStages];
  uint64_t tmem_full;   // P holds a finished chunk
  uint64_t tmem_empty;  // P has been promoted
  uint64_t mma_done;
  uint32_t tmem_base;
  int failed;
  int no_scatter;  // abort fence read at start: scattered rows are not stored
  int issued[kRawStages];
  int prefix[kMaxExperts + 1];
  int scratch[33];
};

constexpr std::size_t kSmemBytes = sizeof(Smem) + 1024;
static_assert(kSmemBytes <= 227 * 1024, "over the 227 KB of shared memory a CTA may use");

// kMT m-tiles of 128 rows share one B tile of 256 / kMT columns (kMT = 2 for
// narrow outputs: the router's N=128 fills the same TMEM and shared memory).
template <int kMT>
__device__ __forceinline__ TileGeom geom(int t, const int32_t* offsets, int experts, int rows,
                                         const int* prefix, int n_tiles_n, int output) {
  return tile_geom(t, offsets, experts, rows, prefix, n_tiles_n, output, kBM * kMT, kBN / kMT);
}

// Element (k, n) of the raw B tile as TMA stores it: N-major, unswizzled,
// 16 rows of kTileN columns (a warp reading 32 consecutive n of one row
// touches 128 contiguous bytes, so the transposing reads are conflict-free).
template <int kTileN>
__device__ __forceinline__ int nmajor_plain_offset(int k, int n) {
  return k * (kTileN * 4) + n * 4;
}

// kGather: A rows come from x through a row map (RowGather) instead of a TMA
// tile of a materialised x_permuted; a separate instantiation so the default
// kernel carries none of it.
// kPrep (prepared expert weights, rr_prepare_expert_weights): B hi and B lo
// arrive K-major from memory (tma_b: W^T, tma_b2: W^T - trunc(W^T)), so the
// MMA takes all of B and A hi from the raw slot and the workers split only
// A. The same shared-memory bytes are cut into 40 KB raw slots (A | B hi |
// B lo) and 8 KB operand slots (A lo).
template <bool kGather, int kMT, bool kPrep = false>
__global__ void __launch_bounds__(kThreads, 1) grouped_gemm_tc_kernel(
    const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
    const __grid_constant__ CUtensorMap tma_b2, const int32_t* __restrict__ offsets,
    float* __restrict__ y, int experts, int rows, int hidden, int output, int wsets,
    unsigned* err, const RowScatter scatter, const RowGather gather) {
  static_assert(kMT == 1 || (kMT == 2 && !kGather), "two m-tiles only for the plain path");
  static_assert(!kPrep || (!kGather && kMT == 1), "prepared weights: plain 128-row tiles");
  // Layout of a raw stage: A (kMT x 8 KB) | B (kTileN columns); of an operand
  // stage: A hi | A lo | B hi | B lo (A hi written only when gathering; else
  // the MMA reads A hi from the raw stage). Both total the same bytes for
  // kMT 1, 2.
  constexpr int kTileN = kBN / kMT;
  constexpr int kAB = kABytes * kMT;
  constexpr int kOBRaw = kAB;
  constexpr int kOAHi = 0;
  constexpr int kOALo = kPrep ? 0 : kAB;
  constexpr int kOBHi = 2 * kAB;
  constexpr int kOBLo = 2 * kAB + kTileN * kBK * 4;
  constexpr int kItems = (kTileN * 4 + kWorkerThreads - 1) / kWorkerThreads;
  static_assert(kOBLo + kTileN * kBK * 4 == kOpBytes && kAB + kTileN * kBK * 4 == kRawBytes,
                "stage layout");
  extern __shared__ uint8_t smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                     ~static_cast<uintptr_t>(1023));
  constexpr int kPrepRaw = kABytes + 2 * kBBytes;  // A | B hi | B lo
  constexpr int kPrepOp = kABytes;                 // A lo
  static_assert(kRawStages * kPrepRaw + kOpStages * kPrepOp <=
                    kRawStages * kRawBytes + kOpStages * kOpBytes,
                "prepared-weight slots fit in the ring bytes");
  // The raw and operand rings are the first members of Smem, back to back.
  uint8_t* const ring = reinterpret_cast<uint8_t*>(&s);
  auto raw_stage = [&](int i) -> uint8_t* {
    return kPrep ? ring + i * kPrepRaw : s.raw[i];
  };
  auto op_stage = [&](int i) -> uint8_t* {
    return kPrep ? ring + kRawStages * kPrepRaw + i * kPrepOp : s.op[i];
  };
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_tiles_n = (output + kTileN - 1) / kTileN;
  const int num_kb = (hidden + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kRawStages; ++i) {
      // Gathering: the producer's expect_tx plus one cp.async arrival per lane.
      mbar_init(&s.raw_full[i], kGather ? 33 : 1);
      mbar_init(&s.raw_empty[i], kGather ? kWorkerWarps : 1);
      s.issued[i] = 0;
    }
    for (int i = 0; i < kOpStages; ++i) {
      mbar_init(&s.op_full[i], kWorkerWarps);
      mbar_init(&s.op_empty[i], 1);
    }
    mbar_init(&s.tmem_full, 1);
    mbar_init(&s.tmem_empty, kWorkerWarps);
    mbar_init(&s.mma_done, 1);
    s.failed = 0;
    s.no_scatter = (scatter.abort != nullptr) ? *scatter.abort : 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&s.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  const int total =
      build_tile_prefix(offsets, experts, rows, kBM * kMT, n_tiles_n, s.prefix, s.scratch);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;
  volatile int* failed = &s.failed;

  if (kGather && warp == 0) {
    // ---------------- producer with row gather (whole warp) ----------------
    // A rows come from x[route[row] / div]: per k-block each lane issues 16
    // cp.async of 16 bytes (instruction j: rows 8j..8j+7, lane l copying
    // chunk l%4 of row 8j + l/4, so a warp instruction fills 512 contiguous
    // bytes), stored unswizzled (row-contiguous, 64 B per row); the workers
    // apply the operand swizzle. Each lane then arrives on raw_full when its
    // copies have landed (32 arrivals + lane 0's expect_tx for B). Rows
    // before 0 (shifted first tile) are not fetched; they feed only output
    // rows that are never stored. Lane 0 waits and issues B by TMA.
    if (lane == 0) tma_prefetch_desc(&tma_b);
    int stage = 0;
    uint32_t phase = 0;
    const int chunk = lane & 3;
    for (int t = blockIdx.x; t < total && !*failed; t += gridDim.x) {
      const TileGeom g = geom<kMT>(t, offsets, experts, rows, s.prefix, n_tiles_n, output);
      int tok[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int row = g.base + 8 * j + (lane >> 2);
        tok[j] = row >= 0 ? __ldg(gather.route + row) / gather.div : -1;
      }
      const uint32_t bbytes = kTileN * kBK * 4;
      for (int kb = 0; kb < num_kb; ++kb) {
        int ok = 1;
        if (lane == 0) ok = mbar_wait(&s.raw_empty[stage], phase ^ 1u, err, failed);
        if (__shfl_sync(0xffffffffu, ok, 0) == 0) break;
        uint8_t* st = s.raw[stage];
        const uint32_t dst = smem_u32(st) + (lane >> 2) * (kBK * 4) + chunk * 16;
        const float* col = gather.x + kb * kBK + chunk * 4;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          if (tok[j] >= 0) {
            cp_async_16(dst + j * 8 * (kBK * 4), col + static_cast<long long>(tok[j]) * hidden);
          }
        }
        cp_async_arrive(&s.raw_full[stage]);
        if (lane == 0) {
          mbar_arrive_expect_tx(&s.raw_full[stage], bbytes);
          tma_load_3d(st + kOBRaw, &tma_b, &s.raw_full[stage], g.col0, kb * kBK,
                      g.expert % wsets);
          s.issued[stage] += 1;
        }
        if (++stage == kRawStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  } else if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      tma_prefetch_desc(&tma_a);
      tma_prefetch_desc(&tma_b);
      if (kPrep) tma_prefetch_desc(&tma_b2);
      int stage = 0;
      uint32_t phase = 0;
      for (int t = blockIdx.x; t < total && !*failed; t += gridDim.x) {
        const TileGeom g = geom<kMT>(t, offsets, experts, rows, s.prefix, n_tiles_n, output);
        // A full-width B box even for a narrow last tile: columns past N
        // are zero-filled by TMA and still count toward the transaction bytes.
        const uint32_t bytes = kPrep ? kPrepRaw : kAB + kTileN * kBK * 4;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&s.raw_empty[stage], phase ^ 1u, err, failed)) break;
          uint8_t* st = raw_stage(stage);
          mbar_arrive_expect_tx(&s.raw_full[stage], bytes);
#pragma unroll
          for (int m = 0; m < kMT; ++m) {
            tma_load_2d(st + m * kABytes, &tma_a, &s.raw_full[stage], kb * kBK, g.base + m * kBM);
          }
          if constexpr (kPrep) {
            // Prepared B tiles: K-major [N][K] per expert, rows past N zero.
            tma_load_3d(st + kABytes, &tma_b, &s.raw_full[stage], kb * kBK, g.col0,
                        g.expert % wsets);
            tma_load_3d(st + kABytes + kBBytes, &tma_b2, &s.raw_full[stage], kb * kBK, g.col0,
                        g.expert % wsets);
          } else {
            tma_load_3d(st + kOBRaw, &tma_b, &s.raw_full[stage], g.col0, kb * kBK,
                        g.expert % wsets);
          }
          s.issued[stage] += 1;
          if (++stage == kRawStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int rstage = 0;
      uint32_t rphase = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total && ok && !*failed; t += gridDim.x) {
        const TileGeom g = geom<kMT>(t, offsets, experts, rows, s.prefix, n_tiles_n, output);
        const uint32_t idesc = idesc_tf32(kBM, g.n_mma, false, false);
        for (int kc = 0; kc < num_kb && ok; kc += kChunkKb) {
          if (!mbar_wait(&s.tmem_empty, acc_phase ^ 1u, err, failed)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // A tile's first chunk accumulates straight into S (it would only
          // be copied there); later chunks go to P and are promoted. Before
          // the second chunk the wait above passes at once (nothing was
          // committed after the first; P is free since the last epilogue).
          const uint32_t d = tmem + (kc == 0 ? kColS : kColP);
          const int kend = min(num_kb, kc + kChunkKb);
          for (int kb = kc; kb < kend; ++kb) {
            if (!mbar_wait(&s.op_full[stage], phase, err, failed) ||
                (!kGather && !mbar_wait(&s.raw_full[rstage], rphase, err, failed))) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t base = smem_u32(op_stage(stage));
            const uint32_t rawb = smem_u32(raw_stage(rstage));
            const uint32_t b_hi = kPrep ? rawb + kABytes : base + kOBHi;
            const uint32_t b_lo = kPrep ? rawb + kABytes + kBBytes : base + kOBLo;
#pragma unroll
            for (int ks = 0; ks < kBK / 8; ++ks) {
              // K-major, 64-byte swizzle: 8-row groups 512 B apart; the second
              // k-step starts 32 B into each row. m-tile m accumulates into
              // TMEM columns m * kTileN.
              const uint64_t bh = smem_desc(b_hi + ks * 32, 16, 512, Swizzle::k64B);
              const uint64_t bl = smem_desc(b_lo + ks * 32, 16, 512, Swizzle::k64B);
              const uint32_t first = (kb == kc && ks == 0) ? 0u : 1u;
#pragma unroll
              for (int m = 0; m < kMT; ++m) {
                const uint32_t a_hi = kGather ? base + kOAHi + m * kABytes : rawb + m * kABytes;
                const uint32_t a_lo = base + kOALo + m * kABytes;
                const uint64_t ah = smem_desc(a_hi + ks * 32, 16, 512, Swizzle::k64B);
                const uint64_t al = smem_desc(a_lo + ks * 32, 16, 512, Swizzle::k64B);
                const uint32_t dm = d + m * kTileN;
                mma_tf32(dm, al, bh, idesc, first);
                mma_tf32(dm, ah, bl, idesc, 1u);
                mma_tf32(dm, ah, bh, idesc, 1u);
              }
            }
            mma_commit(&s.op_empty[stage]);
            if (!kGather) mma_commit(&s.raw_empty[rstage]);
            if (++stage == kOpStages) {
              stage = 0;
              phase ^= 1u;
            }
            if (++rstage == kRawStages) {
              rstage = 0;
              rphase ^= 1u;
            }
          }
          if (!ok) break;
          if (kc == 0 && kend < num_kb) continue;  // no promotion of the first chunk
          mma_commit(&s.tmem_full);
          acc_phase ^= 1u;
        }
      }
      // All MMAs this thread issued are complete once mma_done fires.
      mma_commit(&s.mma_done);
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
    // A chunk of this thread: 16 bytes at tid*16 of the raw tile (row tid/4,
    // chunk tid%4 as TMA stored it, swizzled, or unswizzled when gathered),
    // written to its K-major operand position.
    const uint32_t a_dst = kGather ? static_cast<uint32_t>(kmajor64_offset(tid >> 2, tid & 3))
                                   : static_cast<uint32_t>(tid * 16);
    int rstage = 0, ostage = 0;
    uint32_t rphase = 0, ophase = 0, acc_phase = 0;
    // The chunk awaiting promotion (tile geometry + whether it ends its tile).
    bool pending = false, pending_first = false, pending_last = false;
    TileGeom pg{};
    int t = blockIdx.x;
    int kb = 0;
    TileGeom g{};
    if (t < total) g = geom<kMT>(t, offsets, experts, rows, s.prefix, n_tiles_n, output);
    // This thread's B items (n, kc) of a k-block depend only on the tile's
    // width, so their shared-memory offsets are computed once per tile: item
    // (n, kc) reads rows 4kc..4kc+3 of column n of the N-major raw tile and
    // writes 16 bytes of row n of the K-major operands. A warp covers 32
    // consecutive n of one kc, so the scalar reads are conflict-free and the
    // 16-byte writes take the minimum 4 wavefronts.
    uint32_t bsrc[kItems][4];
    uint32_t bdst[kItems];
    int b_items = 0;
    int b_for = -1;
    auto prepare_b = [&](int n_mma) {
      const int nitems = (((n_mma + 31) >> 5) << 5) * 4;
      b_items = 0;
#pragma unroll
      for (int i = 0; i < kItems; ++i) {
        const int it = tid + i * kWorkerThreads;
        if (it < nitems) b_items = i + 1;
        const int n = (it & 31) + ((it >> 7) << 5);
        const int kc = (it >> 5) & 3;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          bsrc[i][j] = static_cast<uint32_t>(nmajor_plain_offset<kTileN>(4 * kc + j, n));
        }
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
        if (!kPrep && g.n_mma != b_for) prepare_b(g.n_mma);
        const uint32_t raw = smem_u32(raw_stage(rstage));
        const uint32_t op = smem_u32(op_stage(ostage));
        // Loads first (A: one 16-byte chunk in the same K-major position in
        // and out; B: this thread's items), then split and store.
        float4 av[kMT];
#pragma unroll
        for (int m = 0; m < kMT; ++m) av[m] = lds_v4(raw + m * kABytes + tid * 16);
        float4 bv[kItems];
        const uint32_t braw = raw + kOBRaw;
#pragma unroll
        for (int i = 0; i < kItems; ++i) {
          if (!kPrep && i < b_items) {
            bv[i].x = lds_f32(braw + bsrc[i][0]);
            bv[i].y = lds_f32(braw + bsrc[i][1]);
            bv[i].z = lds_f32(braw + bsrc[i][2]);
            bv[i].w = lds_f32(braw + bsrc[i][3]);
          }
        }
        float4 h, l;
#pragma unroll
        for (int m = 0; m < kMT; ++m) {
          // A: hi = v with its low 13 mantissa bits dropped, which is how the
          // MMA reads the raw tile (so without gathering it reads hi straight
          // from the raw slot), lo = v - hi (exact).
          split_trunc4(av[m], h, l);
          if constexpr (kGather) sts_v4(op + kOAHi + m * kABytes + a_dst, h);
          sts_v4(op + kOALo + m * kABytes + a_dst, l);
        }
#pragma unroll
        for (int i = 0; i < kItems; ++i) {
          if (!kPrep && i < b_items) {
            split4(bv[i], h, l);
            sts_v4(op + kOBHi + bdst[i], h);
            sts_v4(op + kOBLo + bdst[i], l);
          }
        }
        // Order this thread's generic reads (raw) and writes (operands)
        // before the async proxy (next TMA into raw, MMA reads of op).
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if (kGather) mbar_arrive(&s.raw_empty[rstage]);
          mbar_arrive(&s.op_full[ostage]);
        }
        if (++rstage == kRawStages) {
          rstage = 0;
          rphase ^= 1u;
        }
        if (++ostage == kOpStages) {
          ostage = 0;
          ophase ^= 1u;
        }
      }
      if (pending) {
        // Promotion of the finished chunk in P.
        if (!mbar_wait(&s.tmem_full, acc_phase, err, failed)) break;
        tc_fence_after();
        // TMEM columns [c_begin, c_begin + 64) of the 256 accumulator
        // columns: m-tile `sub`, output columns from lc0.
        const int c_begin = cgroup * kEpiCols;
        const int sub = c_begin / kTileN;
        const int lc0 = c_begin - sub * kTileN;
        const int row = pg.base + sub * kBM + quarter * 32 + lane;
        bool store_row = pending_last && row >= pg.row0 && row < pg.row_end;
        float* out = y + static_cast<long long>(row) * output + pg.col0 + lc0;
        float wgt = 0.0f;
        if (scatter.dst != nullptr && store_row) {
          float* dst_row = s.no_scatter ? nullptr : scatter_row(scatter, row, output);
          store_row = dst_row != nullptr;
          out = dst_row + pg.col0 + lc0;
        } else if (scatter.combine != nullptr && store_row) {
          out = combine_row(scatter, row, output, wgt) + pg.col0 + lc0;
        }
        // 128-bit stores where the row start allows them (caller-owned
        // scatter bases and combine targets need not be 16-byte aligned).
        const bool vrow = vec && (reinterpret_cast<uintptr_t>(out) & 15) == 0;
        const int w = pg.ncols - lc0;  // columns of this group to store
#pragma unroll
        for (int c = 0; c < kEpiCols; c += 16) {
          if (lc0 + c >= pg.n_mma) break;  // warp-uniform
          const uint32_t col = static_cast<uint32_t>(c_begin + c);
          uint32_t p[16];
          // A first chunk reaches here only when it is also the last: its sum
          // is in S.
          tmem_ld_32x32b_x16(tmem + (pending_first ? kColS : kColP) + col + lane_addr, p);
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
          } else if (store_row && scatter.combine != nullptr) {
            if (vrow) {
#pragma unroll
              for (int j = 0; j < 16; j += 4) {
                if (c + j < w) {
                  red_add_v4_f32(out + c + j, __fmul_rn(wgt, __uint_as_float(p[j])),
                                 __fmul_rn(wgt, __uint_as_float(p[j + 1])),
                                 __fmul_rn(wgt, __uint_as_float(p[j + 2])),
                                 __fmul_rn(wgt, __uint_as_float(p[j + 3])));
                }
              }
            } else {
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                if (c + j < w) red_add_f32(out + c + j, __fmul_rn(wgt, __uint_as_float(p[j])));
              }
            }
          } else if (store_row) {
            if (vrow) {
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
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.tmem_empty);
        acc_phase ^= 1u;
        pending = false;
      }
      if (!have_block) break;
      // A chunk that ends here is promoted next iteration, except a tile's
      // first chunk when more follow (it was accumulated into S directly).
      if (((kb + 1) % kChunkKb == 0 || kb + 1 == num_kb) &&
          !(kb < kChunkKb && kb + 1 < num_kb)) {
        pending = true;
        pending_first = kb < kChunkKb;
        pending_last = (kb + 1 == num_kb);
        pg = g;
      }
      if (++kb == num_kb) {
        kb = 0;
        t += gridDim.x;
        if (t < total) g = geom<kMT>(t, offsets, experts, rows, s.prefix, n_tiles_n, output);
      }
    }
  }

  // Scattered rows may live in another rank's memory: complete those stores
  // before the kernel ends (the barrier that follows publishes them).
  if (scatter.dst != nullptr && warp >= kFirstWorkerWarp) __threadfence_system();
  __syncthreads();
  if (warp == 0 && lane == 0 && *failed) {
    // Drain TMA loads still in flight into this CTA's shared memory.
    for (int i = 0; i < kRawStages; ++i) {
      if (s.issued[i] > 0) {
        int dummy = 0;
        mbar_wait(&s.raw_full[i], static_cast<uint32_t>((s.issued[i] - 1) & 1), err, &dummy);
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---- host side ---------------------------------------------------------------------

EncodeTiledFn encode_fn() { return tensor_map_encoder(); }

bool kernel_configured() {
  static std::once_flag once;
  static bool ok = false;
  std::call_once(once, [] {
    const int bytes = static_cast<int>(kSmemBytes);
    ok = cudaFuncSetAttribute(grouped_gemm_tc_kernel<false, 1>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) == cudaSuccess &&
         cudaFuncSetAttribute(grouped_gemm_tc_kernel<false, 2>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) == cudaSuccess &&
         cudaFuncSetAttribute(grouped_gemm_tc_kernel<true, 1>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) == cudaSuccess &&
         cudaFuncSetAttribute(grouped_gemm_tc_kernel<false, 1, true>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) == cudaSuccess;
    if (!ok) cudaGetLastError();
  });
  return ok;
}

}  // namespace

bool gemm_pairs_enabled() {
  const char* v = std::getenv("RAGGEDROUTE_B200_GEMM_PAIRS");
  return v == nullptr || v[0] != '0';
}

EncodeTiledFn tensor_map_encoder() {
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

cudaError_t launch_grouped_gemm_tc(const float* x, const float* w, const int32_t* offsets,
                                   float* y, int experts, int rows, int hidden, int output,
                                   cudaStream_t stream, int weight_sets,
                                   const RowScatter* scatter, const RowGather* gather) {
  const int wsets = weight_sets > 0 ? weight_sets : experts;
  // One group with at most 128 output columns (the router GEMM): the
  // transposed narrow kernel, at every row count. Its per-element arithmetic
  // (split, K order, promotion) does not depend on the number of rows or on
  // its token-tile height, so a token's logits are the same bits whatever
  // batch it arrives in: a chunked chain (rr_chain_from_tokens_host) equals
  // one chain over the whole batch. (Below two waves of rows the engine
  // would be about as fast, but its bits differ from the narrow kernel's.)
  if (offsets == nullptr && gather == nullptr && scatter == nullptr && output <= kBN / 2 &&
      rows > 0 && dense_narrow_enabled()) {
    const cudaError_t ne = launch_dense_narrow(x, w, y, rows, hidden, output, stream);
    if (ne != cudaErrorNotSupported) return ne;
  }
  EncodeTiledFn encode = encode_fn();
  if (encode == nullptr) return cudaErrorNotSupported;
  if (!kernel_configured()) return cudaErrorNotSupported;
  // A: x [rows, hidden] row-major. Shifted last tiles never read at or past
  // the last segment end, so the row extent only has to cover it.
  const long long a_rows = rows > 0 ? rows : (1LL << 31) - 1;
  CUtensorMap ma{}, mb{};
  if (gather == nullptr) {
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(hidden), static_cast<cuuint64_t>(a_rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(hidden) * 4};
    const cuuint32_t box[2] = {kBK, kBM};
    const cuuint32_t elem[2] = {1, 1};
    if (encode(&ma, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(x), dims, strides, box,
               elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
      return cudaErrorInvalidValue;
    }
  }
  const int mt = (offsets == nullptr && output <= kBN / 2 && gather == nullptr &&
                  scatter == nullptr && rows >= 2LL * kBM * sm_count())
                     ? 2
                     : 1;
  {
    // B: W [experts, hidden, output] viewed as {output, hidden, experts}.
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(output), static_cast<cuuint64_t>(hidden),
                                static_cast<cuuint64_t>(wsets)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(output) * 4,
                                   static_cast<cuuint64_t>(output) * hidden * 4};
    const cuuint32_t box[3] = {static_cast<cuuint32_t>(kBN / mt), kBK, 1};
    const cuuint32_t elem[3] = {1, 1, 1};
    if (encode(&mb, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(w), dims, strides, box,
               elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
      return cudaErrorInvalidValue;
    }
  }
  // One group with at most 128 output columns (the router GEMM) and enough
  // rows to fill every SM with 256-row tiles: two m-tiles per CTA share each
  // B tile (measured at C5: 0.68 -> 0.48 ms). Smaller problems keep 128-row
  // tiles for parallelism.
  int grid = sm_count();
  if (offsets == nullptr) {
    const long long tiles = static_cast<long long>((rows + kBM * mt - 1) / (kBM * mt)) *
                            ((output + kBN / mt - 1) / (kBN / mt));
    if (tiles <= 0) return cudaSuccess;
    if (tiles < grid) grid = static_cast<int>(tiles);
  }
  // The plain path runs on CTA pairs (gemm_pair.cu) wherever the device can
  // co-schedule them; RAGGEDROUTE_B200_GEMM_PAIRS=0 selects this one-CTA
  // kernel instead (both compute the same results).
  if (gather == nullptr && mt == 1 && gemm_pairs_enabled()) {
    const cudaError_t pe = launch_grouped_gemm_pair(x, w, offsets, y, experts, rows, hidden,
                                                    output, stream, weight_sets, scatter);
    if (pe != cudaErrorNotSupported) return pe;
  }
  const RowScatter sc = scatter != nullptr ? *scatter : RowScatter{};
  if (sc.max_ctas > 0 && grid > sc.max_ctas) grid = sc.max_ctas;
  if (gather != nullptr) {
    grouped_gemm_tc_kernel<true, 1><<<grid, kThreads, kSmemBytes, stream>>>(
        ma, mb, mb, offsets, y, experts, rows, hidden, output, wsets, device_error_word(), sc,
        *gather);
  } else if (mt == 2) {
    grouped_gemm_tc_kernel<false, 2><<<grid, kThreads, kSmemBytes, stream>>>(
        ma, mb, mb, offsets, y, experts, rows, hidden, output, wsets, device_error_word(), sc,
        RowGather{});
  } else {
    grouped_gemm_tc_kernel<false, 1><<<grid, kThreads, kSmemBytes, stream>>>(
        ma, mb, mb, offsets, y, experts, rows, hidden, output, wsets, device_error_word(), sc,
        RowGather{});
  }
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_grouped_gemm_prepared(const float* x, const float* w_hi, const float* w_lo,
                                         const int32_t* offsets, float* y, int experts, int rows,
                                         int hidden, int output, cudaStream_t stream,
                                         const RowScatter* scatter) {
  if (hidden <= 0 || output <= 0 || hidden % 4 != 0 || output % 4 != 0 ||
      !aligned_to(x, 16) || !aligned_to(w_hi, 16) || !aligned_to(w_lo, 16) ||
      !aligned_to(y, 16)) {
    return cudaErrorInvalidValue;
  }
  EncodeTiledFn encode = encode_fn();
  if (encode == nullptr || !kernel_configured()) return cudaErrorNotSupported;
  const long long a_rows = rows > 0 ? rows : (1LL << 31) - 1;
  CUtensorMap ma{}, mh{}, ml{};
  {
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(hidden), static_cast<cuuint64_t>(a_rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(hidden) * 4};
    const cuuint32_t box[2] = {kBK, kBM};
    const cuuint32_t elem[2] = {1, 1};
    if (encode(&ma, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(x), dims, strides, box,
               elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
      return cudaErrorInvalidValue;
    }
  }
  // Prepared B: [experts][output][hidden] viewed as {hidden, output, experts},
  // one 16 x 256 box per k-block, K-major with the 64-byte swizzle (the
  // operand layout the MMA reads), rows past N zero-filled.
  for (int i = 0; i < 2; ++i) {
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(hidden), static_cast<cuuint64_t>(output),
                                static_cast<cuuint64_t>(experts)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(hidden) * 4,
                                   static_cast<cuuint64_t>(hidden) * output * 4};
    const cuuint32_t box[3] = {kBK, kBN, 1};
    const cuuint32_t elem[3] = {1, 1, 1};
    if (encode(i == 0 ? &mh : &ml, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3,
               const_cast<float*>(i == 0 ? w_hi : w_lo), dims, strides, box, elem,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
      return cudaErrorInvalidValue;
    }
  }
  int grid = sm_count();
  if (offsets == nullptr) {
    const long long tiles = static_cast<long long>((rows + kBM - 1) / kBM) *
                            ((output + kBN - 1) / kBN);
    if (tiles <= 0) return cudaSuccess;
    if (tiles < grid) grid = static_cast<int>(tiles);
  }
  grouped_gemm_tc_kernel<false, 1, true><<<grid, kThreads, kSmemBytes, stream>>>(
      ma, mh, ml, offsets, y, experts, rows, hidden, output, experts, device_error_word(),
      scatter != nullptr ? *scatter : RowScatter{}, RowGather{});
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_grouped_gemm(const float* x, const float* w, const int32_t* offsets, float* y,
                                int experts, int rows, int hidden, int output,
                                cudaStream_t stream, int weight_sets, const RowScatter* scatter,
                                const RowGather* gather) {
  if (gather != nullptr && (gather->x != x || gather->route == nullptr || gather->div < 1)) {
    return cudaErrorInvalidValue;
  }
  if (tc_gemm_supported(x, w, y, hidden, output)) {
    return launch_grouped_gemm_tc(x, w, offsets, y, experts, rows, hidden, output, stream,
                                  weight_sets, scatter, gather);
  }
  return launch_grouped_gemm_simt(x, w, offsets, y, experts, rows, hidden, output, stream,
                                  weight_sets, scatter, gather);
}

cudaError_t launch_grouped_gemm_combine(const float* x, const float* w, const float* prepared_lo,
                                        const int32_t* offsets, const int32_t* sorted_route,
                                        const float* route_weights, float* y, int experts,
                                        int rows, int tokens, int top_k, int hidden, int output,
                                        cudaStream_t stream, const RowGather* gather) {
  if (top_k < 1 || top_k > 2 || tokens < 0 || output < 0 || rows < 0 ||
      static_cast<long long>(tokens) * top_k < rows) {
    return cudaErrorInvalidValue;
  }
  if (tokens == 0 || output == 0) return cudaSuccess;
  cudaError_t e = cudaMemsetAsync(y, 0, static_cast<std::size_t>(tokens) * output * sizeof(float),
                                  stream);
  if (e != cudaSuccess || rows == 0) return e;
  RowScatter sc;
  sc.combine = y;
  sc.route = sorted_route;
  sc.weight = route_weights;
  sc.top_k = top_k;
  if (prepared_lo != nullptr) {
    return launch_grouped_gemm_prepared(x, w, prepared_lo, offsets, y, experts, rows, hidden,
                                        output, stream, &sc);
  }
  return launch_grouped_gemm(x, w, offsets, y, experts, rows, hidden, output, stream, 0, &sc,
                             gather);
}

}  // namespace rrb
