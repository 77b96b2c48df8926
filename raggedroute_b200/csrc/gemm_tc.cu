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
// below 2^-21 relative per product, far inside the reference's
// accumulation-aware FP32 bound.
//
// Structure: a persistent CTA per SM walks the device-side tile schedule
// (tile_sched.cuh, read from offsets, no host sync). Tiles are 128 rows x 256
// columns; warps are specialised:
//   warp 0     TMA producer: A (x rows, K-major, 64-byte swizzle) and B (the
//              expert's [K, N] weights, N-major, 128-byte swizzle) per 16-wide
//              k-block into a 4-stage ring; no multicast.
//   warps 2-5  split: hi/lo of each landed stage (elementwise, layout-blind).
//   warp 1     MMA issuer: 3 tcgen05.mma (M=128, N<=256, K=8) per k-step into
//              one of two TMEM accumulators (2 x 256 columns), so the epilogue
//              of tile i overlaps the main loop of tile i+1.
//   warps 6-9  epilogue: tcgen05.ld 32 lanes x 32 columns, masked stores.
// A partial last m-tile of an expert is loaded shifted back so it ends at the
// segment end: TMA never reads a row at or beyond offsets[E], and rows before
// the segment come from the previous expert (computed, never stored) or are
// zero-filled when negative. Every mbarrier wait is bounded (2 s); on a timeout
// the kernel records kErrMbarTimeout, drains its own TMA loads and MMAs,
// frees its TMEM and returns.
#include <cuda.h>

#include <mutex>

#include "sm100.cuh"
#include "tile_sched.cuh"

namespace rrb {
namespace {

using namespace sm100;

constexpr int kBM = 128;
constexpr int kBN = 256;
constexpr int kBK = 16;                               // fp32 elements per k-block
constexpr int kStages = 4;
constexpr int kABytes = kBM * kBK * 4;                // 8 KB (64 B rows)
constexpr int kBChunkBytes = 32 * kBK * 4;            // 2 KB: 32 columns x 16 k rows
constexpr int kBBytes = kBN * kBK * 4;                // 16 KB
constexpr int kStageBytes = 2 * (kABytes + kBBytes);  // raw + lo = 48 KB
constexpr int kOffALo = kABytes;
constexpr int kOffBRaw = 2 * kABytes;
constexpr int kOffBLo = 2 * kABytes + kBBytes;
constexpr int kThreads = 320;
constexpr int kTmemCols = 512;
constexpr int kSplitThreads = 128;
constexpr int kEpilogueThreads = 128;

struct alignas(1024) Smem {
  uint8_t stage[kStages][kStageBytes];
  uint64_t full[kStages];
  uint64_t split[kStages];
  uint64_t empty[kStages];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t mma_done;
  uint32_t tmem_base;
  int failed;
  int issued[kStages];
  int prefix[kMaxExperts + 1];
  int scratch[33];
};

constexpr std::size_t kSmemBytes = sizeof(Smem) + 1024;

struct TileGeom {
  int expert, row0, row_end, base, col0, ncols;
};

__device__ __forceinline__ TileGeom geom(int t, const int32_t* offsets, int experts, int rows,
                                         const int* prefix, int n_tiles_n, int output) {
  const TileCoord c = tile_coord(t, offsets, experts, rows, prefix, kBM, kBN, n_tiles_n);
  TileGeom g;
  g.expert = c.expert;
  g.row0 = c.row0;
  g.row_end = c.row_end;
  g.base = (c.row0 + kBM > c.row_end) ? c.row_end - kBM : c.row0;
  g.col0 = c.col0;
  g.ncols = min(kBN, output - c.col0);
  return g;
}

__device__ __forceinline__ void split_vec(float4* raw, float4* lo, int i) {
  const float4 v = raw[i];
  float4 h, l;
  h.x = tf32_rna(v.x);
  h.y = tf32_rna(v.y);
  h.z = tf32_rna(v.z);
  h.w = tf32_rna(v.w);
  l.x = tf32_rna(v.x - h.x);
  l.y = tf32_rna(v.y - h.y);
  l.z = tf32_rna(v.z - h.z);
  l.w = tf32_rna(v.w - h.w);
  raw[i] = h;
  lo[i] = l;
}

__global__ void __launch_bounds__(kThreads, 1) grouped_gemm_tc_kernel(
    const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
    const int32_t* __restrict__ offsets, float* __restrict__ y, int experts, int rows,
    int hidden, int output, unsigned* err) {
  extern __shared__ uint8_t smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                     ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_tiles_n = (output + kBN - 1) / kBN;
  const int num_kb = (hidden + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.split[i], kSplitThreads);
      mbar_init(&s.empty[i], 1);
      s.issued[i] = 0;
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.tmem_full[i], 1);
      mbar_init(&s.tmem_empty[i], kEpilogueThreads);
    }
    mbar_init(&s.mma_done, 1);
    s.failed = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&s.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  const int total =
      build_tile_prefix(offsets, experts, rows, kBM, n_tiles_n, s.prefix, s.scratch);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;
  volatile int* failed = &s.failed;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      tma_prefetch_desc(&tma_a);
      tma_prefetch_desc(&tma_b);
      int stage = 0;
      uint32_t phase = 0;
      for (int t = blockIdx.x; t < total && !*failed; t += gridDim.x) {
        const TileGeom g = geom(t, offsets, experts, rows, s.prefix, n_tiles_n, output);
        const int nchunks = (g.ncols + 31) >> 5;
        const uint32_t bytes = kABytes + nchunks * kBChunkBytes;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&s.empty[stage], phase ^ 1u, err, failed)) break;
          uint8_t* st = s.stage[stage];
          mbar_arrive_expect_tx(&s.full[stage], bytes);
          tma_load_2d(st, &tma_a, &s.full[stage], kb * kBK, g.base);
          for (int j = 0; j < nchunks; ++j) {
            tma_load_3d(st + kOffBRaw + j * kBChunkBytes, &tma_b, &s.full[stage],
                        g.col0 + 32 * j, kb * kBK, g.expert);
          }
          s.issued[stage] += 1;
          if (++stage == kStages) {
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
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int t = blockIdx.x; t < total && !*failed; t += gridDim.x) {
        const TileGeom g = geom(t, offsets, experts, rows, s.prefix, n_tiles_n, output);
        const int n_mma = (g.ncols + 15) & ~15;
        const uint32_t idesc = idesc_tf32(kBM, n_mma, false, true);
        if (!mbar_wait(&s.tmem_empty[acc], acc_phase ^ 1u, err, failed)) break;
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(acc * kBN);
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&s.split[stage], phase, err, failed)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_raw = smem_u32(s.stage[stage]);
          const uint32_t a_lo = a_raw + kOffALo;
          const uint32_t b_raw = a_raw + kOffBRaw;
          const uint32_t b_lo = a_raw + kOffBLo;
#pragma unroll
          for (int ks = 0; ks < kBK / 8; ++ks) {
            const uint64_t ah = smem_desc(a_raw + ks * 32, 16, 512, Swizzle::k64B);
            const uint64_t al = smem_desc(a_lo + ks * 32, 16, 512, Swizzle::k64B);
            const uint64_t bh = smem_desc(b_raw + ks * 1024, kBChunkBytes, 1024, Swizzle::k128B);
            const uint64_t bl = smem_desc(b_lo + ks * 1024, kBChunkBytes, 1024, Swizzle::k128B);
            const uint32_t first = (kb == 0 && ks == 0) ? 0u : 1u;
            mma_tf32(d, al, bh, idesc, first);
            mma_tf32(d, ah, bl, idesc, 1u);
            mma_tf32(d, ah, bh, idesc, 1u);
          }
          mma_commit(&s.empty[stage]);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        mma_commit(&s.tmem_full[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1u;
        }
      }
      // All MMAs this thread issued are complete once mma_done fires.
      mma_commit(&s.mma_done);
      int dummy = 0;
      mbar_wait(&s.mma_done, 0, err, &dummy);
    }
  } else if (warp < 6) {
    // ---------------- hi/lo split ----------------
    const int tid = threadIdx.x - 64;
    int stage = 0;
    uint32_t phase = 0;
    for (int t = blockIdx.x; t < total && !*failed; t += gridDim.x) {
      const TileGeom g = geom(t, offsets, experts, rows, s.prefix, n_tiles_n, output);
      const int nb4 = ((g.ncols + 31) >> 5) * (kBChunkBytes / 16);
      bool ok = true;
      for (int kb = 0; kb < num_kb; ++kb) {
        if (!mbar_wait(&s.full[stage], phase, err, failed)) {
          ok = false;
          break;
        }
        uint8_t* st = s.stage[stage];
        float4* a_raw = reinterpret_cast<float4*>(st);
        float4* a_lo = reinterpret_cast<float4*>(st + kOffALo);
        float4* b_raw = reinterpret_cast<float4*>(st + kOffBRaw);
        float4* b_lo = reinterpret_cast<float4*>(st + kOffBLo);
#pragma unroll
        for (int i = tid; i < kABytes / 16; i += kSplitThreads) split_vec(a_raw, a_lo, i);
        for (int i = tid; i < nb4; i += kSplitThreads) split_vec(b_raw, b_lo, i);
        fence_proxy_async_smem();
        mbar_arrive(&s.split[stage]);
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) break;
    }
  } else {
    // ---------------- epilogue ----------------
    const int quarter = warp & 3;  // TMEM lanes this warp may access
    const int row_in_tile = quarter * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    const bool vec = (output & 3) == 0;
    for (int t = blockIdx.x; t < total && !*failed; t += gridDim.x) {
      const TileGeom g = geom(t, offsets, experts, rows, s.prefix, n_tiles_n, output);
      if (!mbar_wait(&s.tmem_full[acc], acc_phase, err, failed)) break;
      tc_fence_after();
      const int row = g.base + row_in_tile;
      const bool valid = row >= g.row0 && row < g.row_end;
      float* out = y + static_cast<long long>(row) * output + g.col0;
      for (int c0 = 0; c0 < g.ncols; c0 += 32) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem + static_cast<uint32_t>(acc * kBN + c0) +
                               (static_cast<uint32_t>(quarter * 32) << 16),
                           r);
        tmem_ld_wait();
        if (valid) {
          const int w = min(32, g.ncols - c0);
          if (vec) {
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
              if (j < w) {
                *reinterpret_cast<float4*>(out + c0 + j) =
                    make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]),
                                __uint_as_float(r[j + 2]), __uint_as_float(r[j + 3]));
              }
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              if (j < w) out[c0 + j] = __uint_as_float(r[j]);
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&s.tmem_empty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1u;
      }
    }
  }

  __syncthreads();
  if (warp == 0 && lane == 0 && *failed) {
    // Drain TMA loads still in flight into this CTA's shared memory.
    for (int i = 0; i < kStages; ++i) {
      if (s.issued[i] > 0) {
        int dummy = 0;
        mbar_wait(&s.full[i], static_cast<uint32_t>((s.issued[i] - 1) & 1), err, &dummy);
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

bool kernel_configured() {
  static std::once_flag once;
  static bool ok = false;
  std::call_once(once, [] {
    ok = cudaFuncSetAttribute(grouped_gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(kSmemBytes)) == cudaSuccess;
    if (!ok) cudaGetLastError();
  });
  return ok;
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

cudaError_t launch_grouped_gemm_tc(const float* x, const float* w, const int32_t* offsets,
                                   float* y, int experts, int rows, int hidden, int output,
                                   cudaStream_t stream) {
  EncodeTiledFn encode = encode_fn();
  if (encode == nullptr || !kernel_configured()) return cudaErrorNotSupported;
  // A: x [rows, hidden] row-major. Shifted last tiles never read at or past
  // the last segment end, so the row extent only has to cover it.
  const long long a_rows = rows > 0 ? rows : (1LL << 31) - 1;
  CUtensorMap ma{}, mb{};
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
  {
    // B: W [experts, hidden, output] viewed as {output, hidden, experts}.
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(output), static_cast<cuuint64_t>(hidden),
                                static_cast<cuuint64_t>(experts)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(output) * 4,
                                   static_cast<cuuint64_t>(output) * hidden * 4};
    const cuuint32_t box[3] = {32, kBK, 1};
    const cuuint32_t elem[3] = {1, 1, 1};
    if (encode(&mb, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(w), dims, strides, box,
               elem, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
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
  grouped_gemm_tc_kernel<<<grid, kThreads, kSmemBytes, stream>>>(
      ma, mb, offsets, y, experts, rows, hidden, output, device_error_word());
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_grouped_gemm(const float* x, const float* w, const int32_t* offsets, float* y,
                                int experts, int rows, int hidden, int output,
                                cudaStream_t stream) {
  if (tc_gemm_supported(x, w, y, hidden, output)) {
    return launch_grouped_gemm_tc(x, w, offsets, y, experts, rows, hidden, output, stream);
  }
  return launch_grouped_gemm_simt(x, w, offsets, y, experts, rows, hidden, output, stream);
}

}  // namespace rrb
