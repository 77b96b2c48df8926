// Dense GEMM with a narrow output (N <= 128: the router, N = experts) on the
// tcgen05 tensor cores, computed transposed: Y^T = W^T X^T.
//
// Contract: the dense_gemm of src/dense_gemm/cuda_naive/baseline.cu:16-58 of
// the reference, y[m, n] = x[m, :] . w[:, n], with the operand splits of the
// CTA-pair grouped engine (gemm_pair.cu: the mixed split, TF32 hi.hi plus
// bfloat16 corrections, from K = 128 up unless RAGGEDROUTE_B200_GEMM_MIXED=0;
// 3xTF32 below) and the promotion every 512 of K, so the results hold the
// same FP32 contract (not bit-identical to that engine: the tensor core sums
// a product's terms in its own order per M x N shape).
//
// Why transposed: with the expert dimension (128) as the MMA's M, the token
// dimension becomes the MMA's N, which may be any multiple of 16 up to 256.
// The tile height is chosen so that the tiles fill whole waves of SMs (C5:
// 65536 tokens in 293 tiles of 224 for 148 SMs, 99% of two rounds, where the
// engine's 256-row tiles gave 256 tiles, 86% of two rounds), and per k-block
// a CTA splits only a 128-column W tile and its token rows.
//
// Roles (one CTA per SM, persistent over token tiles, 576 threads):
//   warp 0     TMA: x rows (K-major, 64-byte swizzle, TM rows x 16) and the
//              W tile (N-major, unswizzled, 16 x 128, columns past N zero)
//              per 16-wide k-block into a raw ring;
//   warp 1     MMA: per k-step 3 tcgen05.mma (M=128, N=TM, K=8): W^T lo . X
//              hi, W^T hi . X lo, W^T hi . X hi into the TMEM partial P; X hi
//              is the raw tile (the MMA reads FP32 bits as TF32, truncated);
//   warps 2-17 split (W^T hi/lo transposed to K-major, X lo = x - trunc(x))
//              into an operand ring; promotion of P into S every 512 of K;
//              final S + P stored transposed into y (TMEM lane = column n,
//              TMEM column = token; a warp stores 32 consecutive n of a row).
// Every mbarrier wait is bounded (2 s); on a timeout the kernel records
// kErrMbarTimeout, drains its TMA loads and MMAs, frees TMEM and returns.
#include <cuda.h>

#include <cstdlib>
#include <mutex>

#include "gemm_split.cuh"
#include "sm100.cuh"

namespace rrb {
namespace {

using namespace sm100;

constexpr int kNW = 128;                            // W columns per tile (MMA M)
constexpr int kMaxTM = 256;                         // token rows per tile (MMA N), max
constexpr int kBK = 16;                             // fp32 elements per k-block
constexpr int kRawStages = 5;
constexpr int kOpStages = 2;
constexpr int kXBytes = kMaxTM * kBK * 4;           // 16 KB (64 B rows)
constexpr int kWBytes = kNW * kBK * 4;              // 8 KB
constexpr int kRawBytes = kXBytes + kWBytes;        // X raw | W raw (N-major)
constexpr int kOpBytes = kXBytes + 2 * kWBytes;     // X lo | W^T hi | W^T lo
// Mixed split: the operand slot re-cut as W^T hi (TF32) | W^T | W^T lo |
// X | X lo (bfloat16, K-major with the 32-byte swizzle).
constexpr int kOffMWHi = 0;
constexpr int kOffMW = kWBytes;
constexpr int kOffMWLo = kOffMW + kWBytes / 2;
constexpr int kOffMX = 2 * kWBytes;
constexpr int kOffMXLo = kOffMX + kXBytes / 2;
static_assert(kOffMXLo + kXBytes / 2 == kOpBytes, "the mixed split fills the operand slot");
constexpr int kChunkKb = 32;                        // k-blocks per promoted chunk (K = 512)
constexpr uint32_t kColP = 0;
constexpr uint32_t kColS = 256;
constexpr int kWorkerWarps = 16;
constexpr int kFirstWorkerWarp = 2;
constexpr int kThreads = (kFirstWorkerWarp + kWorkerWarps) * 32;  // 576
constexpr int kWorkerThreads = kWorkerWarps * 32;
constexpr int kTmemCols = 512;
constexpr int kEpiCols = kMaxTM / 4;  // token columns per worker thread

struct alignas(1024) NarrowSmem {
  uint8_t raw[kRawStages][kRawBytes];
  uint8_t op[kOpStages][kOpBytes];
  uint64_t raw_full[kRawStages];
  uint64_t raw_empty[kRawStages];
  uint64_t op_full[kOpStages];
  uint64_t op_empty[kOpStages];
  uint64_t tmem_full;
  uint64_t tmem_empty;
  uint64_t mma_done;
  uint32_t tmem_base;
  int failed;
  int issued[kRawStages];
};
constexpr std::size_t kNarrowSmemBytes = sizeof(NarrowSmem) + 1024;
static_assert(kNarrowSmemBytes <= 227 * 1024, "over the 227 KB of shared memory a CTA may use");

// Token tile t: rows [row0, row_end) stored, loaded from base (shifted back
// for a partial last tile so TMA never reads past the last row).
struct NarrowTile {
  int row0, row_end, base;
};

__device__ __forceinline__ NarrowTile narrow_tile(int t, int rows, int tm) {
  NarrowTile g;
  g.row0 = t * tm;
  g.row_end = min(rows, g.row0 + tm);
  g.base = (g.row0 + tm > rows && rows >= tm) ? rows - tm : g.row0;
  return g;
}

template <bool kMixed>
__global__ void __launch_bounds__(kThreads, 1) dense_narrow_kernel(
    const __grid_constant__ CUtensorMap tma_x, const __grid_constant__ CUtensorMap tma_w,
    float* __restrict__ y, int rows, int hidden, int output, int tm, unsigned* err) {
  extern __shared__ uint8_t smem_raw[];
  NarrowSmem& s = *reinterpret_cast<NarrowSmem*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int total = (rows + tm - 1) / tm;
  const int num_kb = (hidden + kBK - 1) / kBK;
  const uint32_t xbytes = static_cast<uint32_t>(tm) * kBK * 4;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kRawStages; ++i) {
      mbar_init(&s.raw_full[i], 1);
      mbar_init(&s.raw_empty[i], 1);
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
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&s.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;
  volatile int* failed = &s.failed;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      tma_prefetch_desc(&tma_x);
      tma_prefetch_desc(&tma_w);
      int stage = 0;
      uint32_t phase = 0;
      for (int t = blockIdx.x; t < total && !*failed; t += gridDim.x) {
        const NarrowTile g = narrow_tile(t, rows, tm);
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&s.raw_empty[stage], phase ^ 1u, err, failed)) break;
          uint8_t* st = s.raw[stage];
          // A full-width W box: columns past N are zero-filled by TMA and
          // count toward the transaction bytes.
          mbar_arrive_expect_tx(&s.raw_full[stage], xbytes + kWBytes);
          tma_load_2d(st, &tma_x, &s.raw_full[stage], kb * kBK, g.base);
          tma_load_2d(st + kXBytes, &tma_w, &s.raw_full[stage], 0, kb * kBK);
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
      int stage = 0, rstage = 0;
      uint32_t phase = 0, rphase = 0, acc_phase = 0;
      bool ok = true;
      const uint32_t idesc = idesc_tf32(kNW, tm, false, false);
      const uint32_t idesc16 = idesc_bf16(kNW, tm);
      for (int t = blockIdx.x; t < total && ok && !*failed; t += gridDim.x) {
        for (int kc = 0; kc < num_kb && ok; kc += kChunkKb) {
          if (!mbar_wait(&s.tmem_empty, acc_phase ^ 1u, err, failed)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int kend = min(num_kb, kc + kChunkKb);
          // A tile's first chunk accumulates straight into S; later chunks
          // go to P and are promoted (see the grouped engine).
          const uint32_t dacc = tmem + (kc == 0 ? kColS : kColP);
          for (int kb = kc; kb < kend; ++kb) {
            if (!mbar_wait(&s.op_full[stage], phase, err, failed) ||
                !mbar_wait(&s.raw_full[rstage], rphase, err, failed)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t op = smem_u32(s.op[stage]);
            const uint32_t raw = smem_u32(s.raw[rstage]);
            if constexpr (kMixed) {
              // hi(W).hi(X) in TF32, then W.lo(X) and lo(W).hi(X) in bfloat16.
#pragma unroll
              for (int ks = 0; ks < kBK / 8; ++ks) {
                const uint64_t wh = smem_desc(op + kOffMWHi + ks * 32, 16, 512, Swizzle::k64B);
                const uint64_t xh = smem_desc(raw + ks * 32, 16, 512, Swizzle::k64B);
                mma_tf32(dacc, wh, xh, idesc, (kb == kc && ks == 0) ? 0u : 1u);
              }
              mma_bf16(dacc, smem_desc(op + kOffMW, 16, 256, Swizzle::k32B),
                       smem_desc(op + kOffMXLo, 16, 256, Swizzle::k32B), idesc16, 1u);
              mma_bf16(dacc, smem_desc(op + kOffMWLo, 16, 256, Swizzle::k32B),
                       smem_desc(op + kOffMX, 16, 256, Swizzle::k32B), idesc16, 1u);
            } else {
#pragma unroll
            for (int ks = 0; ks < kBK / 8; ++ks) {
              // K-major, 64-byte swizzle: 8-row groups 512 B apart; the second
              // k-step starts 32 B into each row.
              const uint64_t wh = smem_desc(op + kXBytes + ks * 32, 16, 512, Swizzle::k64B);
              const uint64_t wl =
                  smem_desc(op + kXBytes + kWBytes + ks * 32, 16, 512, Swizzle::k64B);
              const uint64_t xh = smem_desc(raw + ks * 32, 16, 512, Swizzle::k64B);
              const uint64_t xl = smem_desc(op + ks * 32, 16, 512, Swizzle::k64B);
              const uint32_t first = (kb == kc && ks == 0) ? 0u : 1u;
              mma_tf32(dacc, wl, xh, idesc, first);
              mma_tf32(dacc, wh, xl, idesc, 1u);
              mma_tf32(dacc, wh, xh, idesc, 1u);
            }
            }
            mma_commit(&s.op_empty[stage]);
            mma_commit(&s.raw_empty[rstage]);
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
      mma_commit(&s.mma_done);
      int dummy = 0;
      mbar_wait(&s.mma_done, 0, err, &dummy);
    }
  } else {
    // ---------------- workers: split + promotion + store ----------------
    const int tid = threadIdx.x - kFirstWorkerWarp * 32;  // 0..511
    const int ew = warp - kFirstWorkerWarp;
    const int quarter = warp & 3;  // TMEM lanes (W columns) this warp may access
    const int cgroup = ew >> 2;    // 64-token column group of the tile
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    // W item of this thread: column n of the raw tile, k rows 4kc..4kc+3 (a
    // warp reads 32 consecutive columns of one row: conflict-free), written
    // as 16 bytes of row n of the K-major W^T operands.
    const int wn = (tid & 31) + ((tid >> 7) << 5);
    const int wkc = (tid >> 5) & 3;
    uint32_t wsrc[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) wsrc[j] = static_cast<uint32_t>((4 * wkc + j) * (kNW * 4) + wn * 4);
    const uint32_t wdst = static_cast<uint32_t>(kmajor64_offset(wn, wkc));
    // Mixed split: the same W item as four bfloat16 (8 bytes) in row wn of
    // the 32-byte rows; an X chunk c (row c / 4) likewise.
    const uint32_t wdst16 = static_cast<uint32_t>(kmajor32_offset(wn, wkc >> 1) + ((wkc & 1) << 3));
    auto x16_offset = [](int c) {
      const int r = c >> 2;
      const int kc = (c & 3) ^ ((r >> 1) & 3);  // logical 4-float chunk of the raw row
      return static_cast<uint32_t>(kmajor32_offset(r, kc >> 1) + ((kc & 1) << 3));
    };
    const uint32_t xdst16[2] = {x16_offset(tid), x16_offset(tid + kWorkerThreads)};
    // X chunks of this thread: 16 bytes at tid * 16 and (tid + 512) * 16 of
    // the raw tile, written to the same (swizzled) position of X lo.
    const int xchunks = tm * 4;
    int rstage = 0, ostage = 0;
    uint32_t rphase = 0, ophase = 0, acc_phase = 0;
    bool pending = false, pending_first = false, pending_last = false;
    NarrowTile pg{};
    int t = blockIdx.x;
    int kb = 0;
    NarrowTile g{};
    if (t < total) g = narrow_tile(t, rows, tm);
    while (!*failed) {
      const bool have_block = t < total;
      if (have_block) {
        if (!mbar_wait(&s.raw_full[rstage], rphase, err, failed) ||
            !mbar_wait(&s.op_empty[ostage], ophase ^ 1u, err, failed)) {
          break;
        }
        const uint32_t raw = smem_u32(s.raw[rstage]);
        const uint32_t op = smem_u32(s.op[ostage]);
        const float4 x0 = lds_v4(raw + tid * 16);
        float4 x1 = make_float4(0.f, 0.f, 0.f, 0.f);
        const bool second = tid + kWorkerThreads < xchunks;
        if (second) x1 = lds_v4(raw + (tid + kWorkerThreads) * 16);
        float4 wv;
        wv.x = lds_f32(raw + kXBytes + wsrc[0]);
        wv.y = lds_f32(raw + kXBytes + wsrc[1]);
        wv.z = lds_f32(raw + kXBytes + wsrc[2]);
        wv.w = lds_f32(raw + kXBytes + wsrc[3]);
        float4 h, l;
        if constexpr (kMixed) {
          // X: hi = trunc_tf32(x) is read by the MMA from the raw tile; hi
          // and lo = x - hi (exact) go to the bfloat16 tiles. W: hi =
          // rna_tf32(w) (TF32 tile), w and lo = w - hi (exact) in bfloat16.
          if (tid < xchunks) {
            split_trunc4(x0, h, l);
            sts_v2_u32(op + kOffMX + xdst16[0], bf16x2_rn(h.x, h.y), bf16x2_rn(h.z, h.w));
            sts_v2_u32(op + kOffMXLo + xdst16[0], bf16x2_rn(l.x, l.y), bf16x2_rn(l.z, l.w));
          }
          if (second) {
            split_trunc4(x1, h, l);
            sts_v2_u32(op + kOffMX + xdst16[1], bf16x2_rn(h.x, h.y), bf16x2_rn(h.z, h.w));
            sts_v2_u32(op + kOffMXLo + xdst16[1], bf16x2_rn(l.x, l.y), bf16x2_rn(l.z, l.w));
          }
          h.x = tf32_rna(wv.x);
          h.y = tf32_rna(wv.y);
          h.z = tf32_rna(wv.z);
          h.w = tf32_rna(wv.w);
          sts_v4(op + kOffMWHi + wdst, h);
          sts_v2_u32(op + kOffMW + wdst16, bf16x2_rn(wv.x, wv.y), bf16x2_rn(wv.z, wv.w));
          sts_v2_u32(op + kOffMWLo + wdst16, bf16x2_rn(wv.x - h.x, wv.y - h.y),
                     bf16x2_rn(wv.z - h.z, wv.w - h.w));
        } else {
          if (tid < xchunks) {
            split_trunc4(x0, h, l);
            sts_v4(op + tid * 16, l);
          }
          if (second) {
            split_trunc4(x1, h, l);
            sts_v4(op + (tid + kWorkerThreads) * 16, l);
          }
          split4(wv, h, l);
          sts_v4(op + kXBytes + wdst, h);
          sts_v4(op + kXBytes + kWBytes + wdst, l);
        }
        // Order this thread's generic reads and writes before the async
        // proxy (next TMA into raw, MMA reads of op).
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.op_full[ostage]);
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
        if (!mbar_wait(&s.tmem_full, acc_phase, err, failed)) break;
        tc_fence_after();
        const int c_begin = cgroup * kEpiCols;  // first token column of this thread
        const int n = quarter * 32 + lane;      // output column (W column)
        const bool store_col = pending_last && n < output;
#pragma unroll
        for (int c = 0; c < kEpiCols; c += 16) {
          if (c_begin + c >= tm) break;  // warp-uniform
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
          } else if (store_col) {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int row = pg.base + c_begin + c + j;
              if (row >= pg.row0 && row < pg.row_end) {
                y[static_cast<long long>(row) * output + n] = __uint_as_float(p[j]);
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
        if (t < total) g = narrow_tile(t, rows, tm);
      }
    }
  }

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

bool narrow_configured() {
  static std::once_flag once;
  static bool ok = false;
  std::call_once(once, [] {
    ok = cudaFuncSetAttribute(dense_narrow_kernel<false>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(kNarrowSmemBytes)) == cudaSuccess &&
         cudaFuncSetAttribute(dense_narrow_kernel<true>,
                              cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(kNarrowSmemBytes)) == cudaSuccess;
    if (!ok) cudaGetLastError();
  });
  return ok;
}

}  // namespace

bool dense_narrow_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("RAGGEDROUTE_B200_NARROW_DENSE");
    return v == nullptr || v[0] != '0';
  }();
  return on;
}

cudaError_t launch_dense_narrow(const float* x, const float* w, float* y, int rows, int hidden,
                                int output, cudaStream_t stream) {
  if (rows <= 0 || output <= 0 || output > kNW) return cudaErrorInvalidValue;
  EncodeTiledFn encode = tensor_map_encoder();
  if (encode == nullptr || !narrow_configured()) return cudaErrorNotSupported;
  // Tile height: the smallest multiple of 16 (>= 32) that needs at most one
  // tile per SM when one round of 256-row tiles covers the rows, else at most
  // two tiles per SM, capped at the MMA's 256. A tile costs about the same
  // time at any height (its K loop is bound by the per-k-block hand-off), so
  // fewer rounds win: measured at K=4096, N=128, 8192 / 16384 / 37888 rows
  // 284 / 289 / 309 us with two rounds, 146 / 150 / 185 us with one. The height does not change any result
  // bit (the per-element arithmetic is the same).
  const int sms = sm_count();
  const long long rounds = static_cast<long long>(rows) <= static_cast<long long>(sms) * kMaxTM
                               ? 1
                               : 2;
  long long want = (static_cast<long long>(rows) + rounds * sms - 1) / (rounds * sms);
  int tm = static_cast<int>(((want + 15) / 16) * 16);
  if (tm < 32) tm = 32;
  if (tm > kMaxTM) tm = kMaxTM;
  CUtensorMap mx{}, mw{};
  {
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(hidden), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(hidden) * 4};
    const cuuint32_t box[2] = {kBK, static_cast<cuuint32_t>(tm)};
    const cuuint32_t elem[2] = {1, 1};
    if (encode(&mx, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(x), dims, strides, box,
               elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
      return cudaErrorInvalidValue;
    }
  }
  {
    // W [hidden, output] viewed as {output, hidden}; one box is the whole
    // (padded) width over one k-block.
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(output), static_cast<cuuint64_t>(hidden)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(output) * 4};
    const cuuint32_t box[2] = {kNW, kBK};
    const cuuint32_t elem[2] = {1, 1};
    if (encode(&mw, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(w), dims, strides, box,
               elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
      return cudaErrorInvalidValue;
    }
  }
  const int tiles = (rows + tm - 1) / tm;
  const int grid = tiles < sms ? tiles : sms;
  if (gemm_mixed_split(hidden)) {
    dense_narrow_kernel<true><<<grid, kThreads, kNarrowSmemBytes, stream>>>(
        mx, mw, y, rows, hidden, output, tm, device_error_word());
  } else {
    dense_narrow_kernel<false><<<grid, kThreads, kNarrowSmemBytes, stream>>>(
        mx, mw, y, rows, hidden, output, tm, device_error_word());
  }
  note_launch();
  return cudaGetLastError();
}

}  // namespace rrb
