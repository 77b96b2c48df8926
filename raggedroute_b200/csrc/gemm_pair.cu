// Ragged grouped GEMM on CTA pairs (tcgen05.mma.cta_group::2, sm_100a), with
// the FP32 contract of the one-CTA engine (gemm_tc.cu):
// y[r, :] = x[r, :] . W[e] for r in [offsets[e], offsets[e+1]), rows outside
// every segment untouched; offsets == nullptr is one group of `rows` rows.
//
// Two operand splits, one instantiation each:
// * 3xTF32 (kMixed = false; K < 128, or RAGGEDROUTE_B200_GEMM_MIXED=0): the
//   one-CTA engine's split, lo.hi + hi.lo + hi.hi in TF32, bit-identical to
//   it.
// * mixed (kMixed = true, the default from K = 128 up): hi.hi in TF32 (A hi =
//   trunc_tf32(a), read by the MMA from the raw tile; B hi = rna_tf32(b)),
//   plus two correction products in bfloat16, lo(A).B and hi(A).lo(B), with
//   lo(A) = a - hi(A) and lo(B) = b - hi(B) exact in FP32 and every
//   bfloat16 operand rounded to nearest. A kind::f16 MMA runs at twice the
//   kind::tf32 rate, so the three products cost two TF32 steps of tensor time
//   instead of three (measured at C5: 7.39 -> 6.72 ms per launch). The
//   three products sum every part of a.b; the bfloat16 rounding of the
//   corrections leaves at most about 2^-18 of |a||b| per product (typically
//   far less, with random sign), within the accumulation-aware bound
//   4*K*2^-24 of sums of 128 terms and more, and the chain holds 1e-5
//   normwise against FP64 at C5.
//
// Why pairs. The one-CTA engine moves, per SM and 16-wide k-block of a
// 128 x 256 tile, 24 KB in by TMA, 24 KB through the split's reads, 40 KB of
// split operands out and 72 KB into the tensor core: its shared memory is the
// limit, and a 48 KB operand stage leaves room for only two of them, so the
// split's latency shows between MMAs. A pair computes a 256 x 256 tile: each
// CTA loads its own 128 rows of A and HALF of the tile's 256 B columns, splits
// those, and the even CTA's MMAs (M=256) read both CTAs' shared memory and
// accumulate each CTA's 128 rows in its own TMEM. Per SM that is 16 KB in,
// 16 KB read, 24 KB written and 48 KB into the tensor core for the same
// 128 x 256 outputs, and a 40 KB stage (raw A | raw B half | A lo | B hi half
// | B lo half), so five stages fit.
//
// Roles, per CTA of the pair (576 threads):
//   warp 0     TMA producer: this CTA's 128 A rows (K-major, 64-byte swizzle)
//              and B columns [col0 + rank*n/2, +n/2) of the tile (N-major,
//              unswizzled) per k-block into the stage; no multicast.
//   warp 1     even CTA: MMA issuer, 3 x tcgen05.mma.cta_group::2 (M=256,
//              N=tile width, K=8) per k-step into P (mixed split: 2 TF32
//              K=8 and 2 bfloat16 K=16 per k-block); A hi is the raw A tile
//              itself (the MMA reads FP32 bits as TF32 by truncation). One
//              commit to each CTA's `empty` barrier releases a stage in both,
//              one to each CTA's `tmem_full` hands P to both CTAs' workers.
//              Odd CTA: TMEM allocation only.
//   warps 2-17 workers: split A lo and this CTA's B hi/lo (B transposed to
//              K-major, conflict-free) into the stage, then arrive on the
//              EVEN CTA's op_full (32 arrivals: 16 warps of each CTA); promote
//              P into the running sum S every 512 of K as the one-CTA engine
//              does (except that a tile's first chunk is accumulated into S
//              directly, which saves its copy and one MMA stall per tile;
//              the sums are the same bit for bit), and arrive on the even
//              CTA's tmem_empty. Arrivals
//              on the other CTA's barriers use the default (CTA-scope release)
//              form: a cluster-scope release is a memory barrier per arrival,
//              which measured as the dominant stall.
// Waits are bounded (2 s); a CTA that times out
// records kErrMbarTimeout and sets the failure flag of both CTAs. Before
// either CTA exits, its producer waits until the pair's MMAs released every
// stage it filled (no tensor-core read of, or commit into, an exited CTA's
// shared memory), and both CTAs meet at a cluster barrier before freeing TMEM.
// A 256-row tile pads a ragged expert's last tile further than a 128-row one,
// so a last m-tile that stores at most 128 rows is issued as M = 128 (64 rows
// per CTA, half the tensor-core time); tiles are scheduled on the device from
// offsets (tile_sched.cuh), with the last m-tile of an expert shifted back to
// end at the segment end.
#include <cuda.h>

#include <cstdlib>
#include <mutex>

#include "gemm_split.cuh"
#include "sm100.cuh"
#include "tile_sched.cuh"

namespace rrb {
namespace {

using namespace sm100;

constexpr int kRows = 128;             // A rows per CTA = TMEM lanes
constexpr int kTileM = 2 * kRows;      // output rows per pair tile
constexpr int kTileN = 256;            // output columns per tile
constexpr int kHalfN = kTileN / 2;     // B columns held per CTA
constexpr int kBK = 16;                // fp32 elements per k-block
constexpr int kABytes = kRows * kBK * 4;    // 8 KB
constexpr int kBBytes = kHalfN * kBK * 4;   // 8 KB
constexpr uint32_t kRawTx = kABytes + kBBytes;  // TMA bytes per k-block per CTA
constexpr int kChunkKb = 32;                    // k-blocks per promoted chunk (K = 512)
constexpr uint32_t kColP = 0;                   // TMEM columns of the chunk partial
constexpr uint32_t kColS = kTileN;              // TMEM columns of the running sum
constexpr int kWorkerWarps = 16;
constexpr int kFirstWorkerWarp = 2;
constexpr int kThreads = (kFirstWorkerWarp + kWorkerWarps) * 32;  // 576
constexpr int kTmemCols = 512;
constexpr int kEpiCols = kTileN / 4;  // columns per worker thread in the promotion

// Stage: raw A | raw B half | A lo | B hi half | B lo half (40 KB).
constexpr int kStages = 5;
constexpr int kOffARaw = 0;
constexpr int kOffBRaw = kABytes;
constexpr int kOffALo = 2 * kABytes;
constexpr int kOffBHi = 3 * kABytes;
constexpr int kOffBLo = kOffBHi + kBBytes;
constexpr int kStageBytes = kOffBLo + kBBytes;

// Mixed split (kMixed): the same 40 KB re-cut as raw A | raw B half | B hi
// half (TF32) | A lo | A | B half | B lo half (bfloat16, 4 KB each).
constexpr int kA16Bytes = kRows * kBK * 2;
constexpr int kB16Bytes = kHalfN * kBK * 2;
constexpr int kOffMBHi = 2 * kABytes;
constexpr int kOffMALo = kOffMBHi + kBBytes;
constexpr int kOffMA = kOffMALo + kA16Bytes;
constexpr int kOffMB = kOffMA + kA16Bytes;
constexpr int kOffMBLo = kOffMB + kB16Bytes;
static_assert(kOffMBLo + kB16Bytes == kStageBytes, "the mixed split fills the same stage");
// Below this K the mixed split's per-product error (about 2^-18 of |a||b|
// at worst, from the bfloat16 rounding of the correction operands) could
// exceed the accumulation-aware bound 4*K*2^-24 of short sums; the 3xTF32
// split runs there.
constexpr int kMixedMinK = 128;

struct alignas(1024) PairSmem {
  uint8_t stage[kStages][kStageBytes];
  uint64_t raw_full[kStages];  // this CTA's TMA bytes of the stage landed
  uint64_t empty[kStages];     // the pair's MMAs finished reading the stage
  uint64_t op_full[kStages];   // even CTA: both CTAs' workers split the stage
  uint64_t tmem_full;          // P holds a finished chunk (both CTAs)
  uint64_t tmem_empty;         // even CTA: both CTAs promoted P
  uint64_t mma_done;
  uint32_t tmem_base;
  int failed;
  int no_scatter;  // abort fence read at start: scattered rows are not stored
  int issued[kStages];
  int prefix[kMaxExperts + 1];
  int scratch[33];
};
constexpr std::size_t kPairSmemBytes = sizeof(PairSmem) + 1024;
static_assert(kPairSmemBytes <= 227 * 1024, "over the 227 KB of shared memory a CTA may use");
static_assert(kStageBytes % 1024 == 0, "stages keep the 1 KB alignment of the swizzled tiles");

template <bool kMixed>
__global__ void __launch_bounds__(kThreads, 1) grouped_gemm_pair_kernel(
    const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
    const int32_t* __restrict__ offsets, float* __restrict__ y, int experts, int rows,
    int hidden, int output, int wsets, unsigned* err, const RowScatter scatter) {
  extern __shared__ uint8_t smem_raw[];
  PairSmem& s = *reinterpret_cast<PairSmem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int unit = static_cast<int>(blockIdx.x >> 1);
  const int units = static_cast<int>(gridDim.x >> 1);
  const int n_tiles_n = (output + kTileN - 1) / kTileN;
  const int num_kb = (hidden + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&s.raw_full[i], 1);
      mbar_init(&s.empty[i], 1);
      mbar_init(&s.op_full[i], 2 * kWorkerWarps);
      s.issued[i] = 0;
    }
    mbar_init(&s.tmem_full, 1);
    mbar_init(&s.tmem_empty, 2 * kWorkerWarps);
    mbar_init(&s.mma_done, 1);
    s.failed = 0;
    s.no_scatter = (scatter.abort != nullptr) ? *scatter.abort : 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(&s.tmem_base, kTmemCols);
    tmem_relinquish_pair();
  }
  const int total =
      build_tile_prefix(offsets, experts, rows, kTileM, n_tiles_n, s.prefix, s.scratch);
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers are initialised and TMEM allocated
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;
  volatile int* failed = &s.failed;
  const uint32_t peer_failed = mapa_shared(smem_u32(&s.failed), rank ^ 1u);
  auto wait = [&](uint64_t* bar, uint32_t parity) {
    return mbar_wait_pair(bar, parity, err, failed, peer_failed);
  };
  auto geom = [&](int t) {
    return tile_geom(t, offsets, experts, rows, s.prefix, n_tiles_n, output, kTileM, kTileN, true);
  };

  if (warp == 0) {
    // ---------------- TMA producer: this CTA's A rows and B columns ----------------
    if (lane == 0) {
      tma_prefetch_desc(&tma_a);
      tma_prefetch_desc(&tma_b);
      int stage = 0;
      uint32_t phase = 0;
      for (int t = unit; t < total && !*failed; t += units) {
        const TileGeom g = geom(t);
        // CTA r holds rows [r*m/2, (r+1)*m/2) of the tile (m = 256, or 128
        // for a half tail tile, of whose 128-row box the MMA reads the first
        // 64 rows).
        const int arow = g.base + static_cast<int>(rank) * (g.m_mma >> 1);
        const int bcol = g.col0 + static_cast<int>(rank) * (g.n_mma >> 1);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!wait(&s.empty[stage], phase ^ 1u)) break;
          uint8_t* st = s.stage[stage];
          // A full 128-column B box even when this CTA uses fewer columns:
          // columns past N are zero-filled and count toward the bytes.
          mbar_arrive_expect_tx(&s.raw_full[stage], kRawTx);
          tma_load_2d(st + kOffARaw, &tma_a, &s.raw_full[stage], kb * kBK, arow);
          tma_load_3d(st + kOffBRaw, &tma_b, &s.raw_full[stage], bcol, kb * kBK,
                      g.expert % wsets);
          s.issued[stage] += 1;
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Tail: wait until the pair's MMAs have released every stage (their
      // last use), so nothing reads or signals this CTA's shared memory
      // after it exits.
      for (int i = 0; i < kStages && !*failed; ++i) {
        if (!wait(&s.empty[stage], phase ^ 1u)) break;
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (even CTA) ----------------
    if (leader && lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      const uint32_t tmem_full_local = smem_u32(&s.tmem_full);
      const uint32_t tmem_full_peer = mapa_shared(tmem_full_local, 1u);
      for (int t = unit; t < total && ok && !*failed; t += units) {
        const TileGeom g = geom(t);
        const uint32_t idesc = idesc_tf32(g.m_mma, g.n_mma, false, false);
        const uint32_t idesc16 = idesc_bf16(g.m_mma, g.n_mma);
        for (int kc = 0; kc < num_kb && ok; kc += kChunkKb) {
          if (!wait(&s.tmem_empty, acc_phase ^ 1u)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // Every chunk accumulates into P and is promoted into S (a tile's
          // first chunk by a copy). P is free once the previous chunk's
          // promotion has read it; the previous tile's stores from S then
          // run beside this chunk's MMAs.
          const uint32_t d = tmem + kColP;
          const int kend = min(num_kb, kc + kChunkKb);
          for (int kb = kc; kb < kend; ++kb) {
            if (!wait(&s.op_full[stage], phase)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t base = smem_u32(s.stage[stage]);
            if constexpr (kMixed) {
              // hi.hi in TF32 (two K=8 steps), then the corrections lo(A).B
              // and A.lo(B) in bfloat16 (one K=16 step each, at twice the
              // TF32 rate): two TF32 steps' worth of tensor time, not three.
#pragma unroll
              for (int ks = 0; ks < kBK / 8; ++ks) {
                const uint64_t ah =
                    smem_desc(base + kOffARaw + ks * 32, 16, 512, Swizzle::k64B);
                const uint64_t bh =
                    smem_desc(base + kOffMBHi + ks * 32, 16, 512, Swizzle::k64B);
                mma_tf32_pair(d, ah, bh, idesc, (kb == kc && ks == 0) ? 0u : 1u);
              }
              // 32-byte rows, 8-row groups 256 B apart.
              mma_bf16_pair(d, smem_desc(base + kOffMALo, 16, 256, Swizzle::k32B),
                            smem_desc(base + kOffMB, 16, 256, Swizzle::k32B), idesc16, 1u);
              mma_bf16_pair(d, smem_desc(base + kOffMA, 16, 256, Swizzle::k32B),
                            smem_desc(base + kOffMBLo, 16, 256, Swizzle::k32B), idesc16, 1u);
            } else {
#pragma unroll
            for (int ks = 0; ks < kBK / 8; ++ks) {
              // K-major, 64-byte swizzle: 8-row groups 512 B apart; the
              // second k-step starts 32 B into each row.
              const uint64_t bh = smem_desc(base + kOffBHi + ks * 32, 16, 512, Swizzle::k64B);
              const uint64_t bl = smem_desc(base + kOffBLo + ks * 32, 16, 512, Swizzle::k64B);
              const uint32_t first = (kb == kc && ks == 0) ? 0u : 1u;
              const uint64_t ah =
                  smem_desc(base + kOffARaw + ks * 32, 16, 512, Swizzle::k64B);
              const uint64_t al =
                  smem_desc(base + kOffALo + ks * 32, 16, 512, Swizzle::k64B);
              mma_tf32_pair(d, al, bh, idesc, first);
              mma_tf32_pair(d, ah, bl, idesc, 1u);
              mma_tf32_pair(d, ah, bh, idesc, 1u);
            }
            }
            const uint32_t e = smem_u32(&s.empty[stage]);
            mma_commit_pair_to(e);
            mma_commit_pair_to(mapa_shared(e, 1u));
            if (++stage == kStages) {
              stage = 0;
              phase ^= 1u;
            }
          }
          if (!ok) break;
          mma_commit_pair_to(tmem_full_local);
          mma_commit_pair_to(tmem_full_peer);
          acc_phase ^= 1u;
        }
      }
      // All MMAs this thread issued are complete once mma_done fires.
      mma_commit_pair_to(smem_u32(&s.mma_done));
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
    const uint32_t op_full_leader = mapa_shared(smem_u32(&s.op_full[0]), 0u);
    const uint32_t tmem_empty_leader = mapa_shared(smem_u32(&s.tmem_empty), 0u);
    // This thread's B item: column bn of this CTA's half, k rows 4*bkc..+3.
    // A warp covers 32 consecutive columns of one bkc: the four scalar reads
    // each touch 128 contiguous bytes and the 16-byte writes take the
    // minimum four wavefronts.
    const int bn = (tid & 31) + ((tid >> 7) << 5);
    const int bkc = (tid >> 5) & 3;
    uint32_t bsrc[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) bsrc[j] = static_cast<uint32_t>((4 * bkc + j) * (kHalfN * 4) + bn * 4);
    const uint32_t bdst = static_cast<uint32_t>(kmajor64_offset(bn, bkc));
    // Mixed split: worker warps 0-7 take B (column mbn of this CTA's half, k
    // rows 8*mkh..+7: eight 128-byte row reads per warp, 16-byte bfloat16
    // chunks that fill all 32 banks), warps 8-15 take A (the 16-byte chunks
    // ca and ca + 256 of the raw tile, each written as two 8-byte bfloat16
    // halves at the same row and k of the 32-byte-swizzled tiles).
    const int mbn = (tid & 31) + ((ew >> 1) << 5);
    const int mkh = ew & 1;
    const uint32_t mb_src = static_cast<uint32_t>(8 * mkh * (kHalfN * 4) + mbn * 4);
    const uint32_t mb_hi0 = static_cast<uint32_t>(kmajor64_offset(mbn, 2 * mkh));
    const uint32_t mb_hi1 = static_cast<uint32_t>(kmajor64_offset(mbn, 2 * mkh + 1));
    const uint32_t mb_16 = static_cast<uint32_t>(kmajor32_offset(mbn, mkh));
    const int ca = tid & 255;
    auto a16_offset = [](int c) {
      const int r = c >> 2;
      const int kc = (c & 3) ^ ((r >> 1) & 3);  // logical 4-float chunk of the raw row
      return static_cast<uint32_t>(kmajor32_offset(r, kc >> 1) + ((kc & 1) << 3));
    };
    const uint32_t ma_16[2] = {a16_offset(ca), a16_offset(ca + 256)};
    int stage = 0;
    uint32_t phase = 0, acc_phase = 0;
    bool pending = false, pending_first = false, pending_last = false;
    // Stores of a finished tile's y from S still to do: the next column
    // offset within this thread's 64 columns, or -1.
    int epi_c = -1, epi_cb = 0, epi_width = 0, epi_w = 0;
    bool epi_store = false, epi_vrow = false;
    float* epi_out = nullptr;
    float epi_wgt = 0.0f;
    auto epi_step = [&]() {
      const int c = epi_c;
      uint32_t p[16];
      tmem_ld_32x32b_x16(tmem + kColS + static_cast<uint32_t>(epi_cb + c) + lane_addr, p);
      tmem_ld_wait();
      float* const out = epi_out;
      const int w = epi_w;
      if (epi_store && scatter.combine != nullptr) {
        if (epi_vrow) {
#pragma unroll
          for (int j = 0; j < 16; j += 4) {
            if (c + j < w) {
              red_add_v4_f32(out + c + j, __fmul_rn(epi_wgt, __uint_as_float(p[j])),
                             __fmul_rn(epi_wgt, __uint_as_float(p[j + 1])),
                             __fmul_rn(epi_wgt, __uint_as_float(p[j + 2])),
                             __fmul_rn(epi_wgt, __uint_as_float(p[j + 3])));
            }
          }
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            if (c + j < w) red_add_f32(out + c + j, __fmul_rn(epi_wgt, __uint_as_float(p[j])));
          }
        }
      } else if (epi_store) {
        if (epi_vrow) {
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
      epi_c = c + 16;
      if (epi_c >= kEpiCols || epi_cb + epi_c >= epi_width) epi_c = -1;  // warp-uniform
    };
    TileGeom pg{};
    int t = unit;
    int kb = 0;
    TileGeom g{};
    if (t < total) g = geom(t);
    // One iteration = split one k-block (while any remain), then promote the
    // previously finished chunk. A final iteration without a k-block drains
    // the last chunk.
    while (!*failed) {
      const bool have_block = t < total;
      if (have_block) {
        if (!wait(&s.raw_full[stage], phase)) break;
        const uint32_t st = smem_u32(s.stage[stage]);
        if constexpr (kMixed) {
          if (ew < 8) {
            // B: hi = rna_tf32(v) for the TF32 product; v and lo = v - hi
            // (exact) rounded to bfloat16 for the correction products.
            if (mbn < (((g.n_mma >> 1) + 31) & ~31)) {  // warp-uniform
              float v[8], hi[8];
              uint32_t p16[4], l16[4];
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                v[j] = lds_f32(st + kOffBRaw + mb_src + j * (kHalfN * 4));
                hi[j] = tf32_rna(v[j]);
              }
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                p16[j] = bf16x2_rn(v[2 * j], v[2 * j + 1]);
                l16[j] = bf16x2_rn(v[2 * j] - hi[2 * j], v[2 * j + 1] - hi[2 * j + 1]);
              }
              sts_v4(st + kOffMBHi + mb_hi0, make_float4(hi[0], hi[1], hi[2], hi[3]));
              sts_v4(st + kOffMBHi + mb_hi1, make_float4(hi[4], hi[5], hi[6], hi[7]));
              sts_v4_u32(st + kOffMB + mb_16, p16[0], p16[1], p16[2], p16[3]);
              sts_v4_u32(st + kOffMBLo + mb_16, l16[0], l16[1], l16[2], l16[3]);
            }
          } else {
            // A: the MMA reads hi = trunc_tf32(v) from the raw tile; lo = v -
            // hi (exact) and hi itself go to the bfloat16 tiles, so that
            // hi.hi + lo(A).B + hi(A).lo(B) sums every part of the product.
#pragma unroll
            for (int i = 0; i < 2; ++i) {
              const float4 av = lds_v4(st + kOffARaw + (ca + 256 * i) * 16);
              float4 h, l;
              split_trunc4(av, h, l);
              sts_v2_u32(st + kOffMALo + ma_16[i], bf16x2_rn(l.x, l.y), bf16x2_rn(l.z, l.w));
              sts_v2_u32(st + kOffMA + ma_16[i], bf16x2_rn(h.x, h.y), bf16x2_rn(h.z, h.w));
            }
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive_remote(op_full_leader + stage * 8);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        } else {
        // Columns of this CTA's half that the MMA reads (warp-uniform test).
        const bool b_used = bn < (((g.n_mma >> 1) + 31) & ~31);
        const float4 av = lds_v4(st + kOffARaw + tid * 16);
        float4 bv = make_float4(0.f, 0.f, 0.f, 0.f);
        if (b_used) {
          bv.x = lds_f32(st + kOffBRaw + bsrc[0]);
          bv.y = lds_f32(st + kOffBRaw + bsrc[1]);
          bv.z = lds_f32(st + kOffBRaw + bsrc[2]);
          bv.w = lds_f32(st + kOffBRaw + bsrc[3]);
        }
        float4 h, l;
        split_trunc4(av, h, l);
        // The MMA reads hi (truncated) straight from the raw tile; lo =
        // v - hi goes to the same swizzled position of the A lo tile.
        sts_v4(st + kOffALo + tid * 16, l);
        if (b_used) {
          split4(bv, h, l);
          sts_v4(st + kOffBHi + bdst, h);
          sts_v4(st + kOffBLo + bdst, l);
        }
        // Order this thread's shared-memory writes before the tensor core's
        // reads (async proxy), then hand the stage to the even CTA's MMA.
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(op_full_leader + stage * 8);
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1u;
        }
        }
      }
      if (pending) {
        // Promotion of the finished chunk in P (this CTA's 128 rows): S = P
        // for a tile's first chunk, else S += P, in TMEM only; then P is
        // released to the MMA. For a tile's last chunk the stores of y from
        // S follow, one 16-column group per later iteration (epi_step).
        while (epi_c >= 0) epi_step();  // this thread's reads of S come first
        if (!wait(&s.tmem_full, acc_phase)) break;
        tc_fence_after();
        // A full tile holds this CTA's 128 rows x n_mma columns in TMEM lanes
        // 0-127. A half tile (M = 128: 64 rows per CTA) is folded: lanes 0-63
        // hold columns [0, n_mma/2) of the 64 rows, lanes 64-127 columns
        // [n_mma/2, n_mma), in TMEM columns [0, n_mma/2). Either way thread
        // (quarter, cgroup) owns TMEM lanes quarter*32.. and columns
        // cgroup*64..+63, so every TMEM word of P and S is read and written
        // by one thread only, in program order.
        const bool half = pg.m_mma < kTileM;
        const int width = half ? (pg.n_mma >> 1) : pg.n_mma;  // TMEM columns in use
        const int c_begin = cgroup * kEpiCols;
#pragma unroll
        for (int c = 0; c < kEpiCols; c += 16) {
          if (c_begin + c >= width) break;  // warp-uniform
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
          tmem_st_32x32b_x16(tmem + kColS + col + lane_addr, p);
        }
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(tmem_empty_leader);
        acc_phase ^= 1u;
        if (pending_last && c_begin < width) {
          const int col_base = half ? (quarter >> 1) * width : 0;
          const int row = pg.base + static_cast<int>(rank) * (pg.m_mma >> 1) +
                          (half ? (quarter & 1) * 32 : quarter * 32) + lane;
          bool store_row = row >= pg.row0 && row < pg.row_end;
          float* out = y + static_cast<long long>(row) * output + pg.col0 + col_base + c_begin;
          float wgt = 0.0f;
          if (scatter.dst != nullptr && store_row) {
            float* dst_row = s.no_scatter ? nullptr : scatter_row(scatter, row, output);
            store_row = dst_row != nullptr;
            out = dst_row + pg.col0 + col_base + c_begin;
          } else if (scatter.combine != nullptr && store_row) {
            out = combine_row(scatter, row, output, wgt) + pg.col0 + col_base + c_begin;
          }
          epi_c = 0;
          epi_cb = c_begin;
          epi_width = width;
          epi_store = store_row;
          epi_out = out;
          epi_wgt = wgt;
          // 128-bit stores where the row start allows them (caller-owned
          // scatter bases and combine targets need not be 16-byte aligned).
          epi_vrow = vec && (reinterpret_cast<uintptr_t>(out) & 15) == 0;
          // Columns of this group to store.
          epi_w = min(width, pg.ncols - col_base) - c_begin;
        }
        pending = false;
      } else if (epi_c >= 0) {
        epi_step();
      }
      if (!have_block) {
        while (epi_c >= 0) epi_step();
        break;
      }
      // A chunk that ends here is promoted next iteration.
      if ((kb + 1) % kChunkKb == 0 || kb + 1 == num_kb) {
        pending = true;
        pending_first = kb < kChunkKb;
        pending_last = (kb + 1 == num_kb);
        pg = g;
      }
      if (++kb == num_kb) {
        kb = 0;
        t += units;
        if (t < total) g = geom(t);
      }
    }
  }

  // Scattered rows may live in another rank's memory: complete those stores
  // before the kernel ends (the barrier that follows publishes them).
  if (scatter.dst != nullptr && warp >= kFirstWorkerWarp) __threadfence_system();
  __syncthreads();
  if (warp == 0 && lane == 0 && *failed) {
    // Drain TMA loads still in flight into this CTA's shared memory.
    for (int i = 0; i < kStages; ++i) {
      if (s.issued[i] > 0) {
        int dummy = 0;
        mbar_wait(&s.raw_full[i], static_cast<uint32_t>((s.issued[i] - 1) & 1), err, &dummy);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the pair's MMAs are done; no arrivals into either CTA remain
  tc_fence_after();
  if (warp == 1) tmem_dealloc_pair(tmem, kTmemCols);
}

bool pair_kernel_configured() {
  static std::once_flag once;
  static bool ok = false;
  std::call_once(once, [] {
    ok = cudaFuncSetAttribute(grouped_gemm_pair_kernel<false>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(kPairSmemBytes)) == cudaSuccess &&
         cudaFuncSetAttribute(grouped_gemm_pair_kernel<true>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(kPairSmemBytes)) == cudaSuccess;
    if (!ok) cudaGetLastError();
  });
  return ok;
}

cudaLaunchConfig_t pair_config(int units, cudaStream_t stream, cudaLaunchAttribute* attr) {
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(2 * units, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = kPairSmemBytes;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cfg;
}

}  // namespace

bool gemm_mixed_split(int hidden) {
  static const bool enabled = [] {
    const char* v = std::getenv("RAGGEDROUTE_B200_GEMM_MIXED");
    return v == nullptr || v[0] != '0';
  }();
  return enabled && hidden >= kMixedMinK;
}

int grouped_gemm_pair_units() {
  static std::once_flag once;
  static int units = 0;
  std::call_once(once, [] {
    if (!pair_kernel_configured()) return;
    cudaLaunchAttribute attr[1];
    const cudaLaunchConfig_t cfg = pair_config(sm_count(), nullptr, attr);
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, grouped_gemm_pair_kernel<false>, &cfg) !=
        cudaSuccess) {
      cudaGetLastError();
      n = 0;
    }
    units = n;
  });
  return units;
}

cudaError_t launch_grouped_gemm_pair(const float* x, const float* w, const int32_t* offsets,
                                     float* y, int experts, int rows, int hidden, int output,
                                     cudaStream_t stream, int weight_sets,
                                     const RowScatter* scatter) {
  const int wsets = weight_sets > 0 ? weight_sets : experts;
  EncodeTiledFn encode = tensor_map_encoder();
  int units = grouped_gemm_pair_units();
  if (encode == nullptr || units <= 0) return cudaErrorNotSupported;
  // A: x [rows, hidden] row-major, one CTA's 128 rows per box. Shifted last
  // tiles read no row of a full tile at or past the last segment end; the
  // odd CTA's box of a half tile may reach past `rows` (zero-filled, and
  // beyond the 64 rows its MMA reads).
  const long long a_rows = rows > 0 ? rows : (1LL << 31) - 1;
  CUtensorMap ma{}, mb{};
  {
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(hidden), static_cast<cuuint64_t>(a_rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(hidden) * 4};
    const cuuint32_t box[2] = {kBK, kRows};
    const cuuint32_t elem[2] = {1, 1};
    if (encode(&ma, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(x), dims, strides, box,
               elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
      return cudaErrorInvalidValue;
    }
  }
  {
    // B: W [experts, hidden, output] viewed as {output, hidden, experts}; one
    // box is half a tile's columns over one k-block.
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(output), static_cast<cuuint64_t>(hidden),
                                static_cast<cuuint64_t>(wsets)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(output) * 4,
                                   static_cast<cuuint64_t>(output) * hidden * 4};
    const cuuint32_t box[3] = {kHalfN, kBK, 1};
    const cuuint32_t elem[3] = {1, 1, 1};
    if (encode(&mb, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(w), dims, strides, box,
               elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
      return cudaErrorInvalidValue;
    }
  }
  if (offsets == nullptr) {
    const long long tiles = static_cast<long long>((rows + kTileM - 1) / kTileM) *
                            ((output + kTileN - 1) / kTileN);
    if (tiles <= 0) return cudaSuccess;
    if (tiles < units) units = static_cast<int>(tiles);
  }
  const RowScatter sc = scatter != nullptr ? *scatter : RowScatter{};
  if (sc.max_ctas > 0 && units > sc.max_ctas / 2) units = sc.max_ctas / 2 > 0 ? sc.max_ctas / 2 : 1;
  cudaLaunchAttribute attr[1];
  const cudaLaunchConfig_t cfg = pair_config(units, stream, attr);
  const cudaError_t e =
      gemm_mixed_split(hidden)
          ? cudaLaunchKernelEx(&cfg, grouped_gemm_pair_kernel<true>, ma, mb, offsets, y, experts,
                               rows, hidden, output, wsets, device_error_word(), sc)
          : cudaLaunchKernelEx(&cfg, grouped_gemm_pair_kernel<false>, ma, mb, offsets, y,
                               experts, rows, hidden, output, wsets, device_error_word(), sc);
  if (e != cudaSuccess) return e;
  note_launch();
  return cudaGetLastError();
}

}  // namespace rrb
