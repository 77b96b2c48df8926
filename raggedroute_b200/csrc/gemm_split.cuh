// Pieces shared by the tcgen05 GEMM kernels (gemm_tc.cu: one CTA per tile;
// gemm_pair.cu: a CTA pair per tile): the 3xTF32 operand split, the K-major
// 64-byte-swizzled operand layout, and the geometry of a scheduled tile.
#pragma once

#include "sm100.cuh"
#include "tile_sched.cuh"

namespace rrb {

struct TileGeom {
  int expert, row0, row_end, base, col0, ncols, n_mma, m_mma;
};

// Geometry of tile t of a schedule with tile_m x tile_n tiles. A partial last
// m-tile of an expert is shifted back to end at the segment end (base), so
// TMA never reads a row at or beyond offsets[E]; rows before row0 are
// computed but not stored. n_mma is the tile's width rounded up to 16.
// m_mma is the tile's height: tile_m, or tile_m / 2 for a last m-tile that
// stores at most tile_m / 2 rows when half_tail is set (the CTA-pair engine's
// M = 128 instruction).
__device__ __forceinline__ TileGeom tile_geom(int t, const int32_t* offsets, int experts, int rows,
                                              const int* prefix, int n_tiles_n, int output,
                                              int tile_m, int tile_n, bool half_tail = false) {
  const TileCoord c = tile_coord(t, offsets, experts, rows, prefix, tile_m, tile_n, n_tiles_n);
  TileGeom g;
  g.expert = c.expert;
  g.row0 = c.row0;
  g.row_end = c.row_end;
  g.m_mma = (half_tail && c.row_end - c.row0 <= tile_m / 2) ? tile_m / 2 : tile_m;
  g.base = (c.row0 + g.m_mma > c.row_end) ? c.row_end - g.m_mma : c.row0;
  g.col0 = c.col0;
  g.ncols = min(tile_n, output - c.col0);
  g.n_mma = (g.ncols + 15) & ~15;
  return g;
}

// B operand split: hi = rna_tf32(v), lo = rna_tf32(v - hi).
__device__ __forceinline__ void split4(const float4 v, float4& h, float4& l) {
  h.x = sm100::tf32_rna(v.x);
  h.y = sm100::tf32_rna(v.y);
  h.z = sm100::tf32_rna(v.z);
  h.w = sm100::tf32_rna(v.w);
  l.x = sm100::tf32_rna(v.x - h.x);
  l.y = sm100::tf32_rna(v.y - h.y);
  l.z = sm100::tf32_rna(v.z - h.z);
  l.w = sm100::tf32_rna(v.w - h.w);
}

// A operand split: hi = v with the low 13 mantissa bits cleared (the value
// a kind::tf32 MMA reads from the raw FP32 bits), lo = v - hi (exact in FP32,
// up to 13 significant bits, of which the MMA keeps the top 11).
__device__ __forceinline__ void split_trunc4(const float4 v, float4& h, float4& l) {
  h.x = __uint_as_float(__float_as_uint(v.x) & 0xFFFFE000u);
  h.y = __uint_as_float(__float_as_uint(v.y) & 0xFFFFE000u);
  h.z = __uint_as_float(__float_as_uint(v.z) & 0xFFFFE000u);
  h.w = __uint_as_float(__float_as_uint(v.w) & 0xFFFFE000u);
  l.x = v.x - h.x;
  l.y = v.y - h.y;
  l.z = v.z - h.z;
  l.w = v.w - h.w;
}

// Byte offset of 16-byte chunk kc (k = 4*kc..4*kc+3) of row r in a K-major
// tile of 16 fp32 per row with the 64-byte swizzle (TMA and UMMA agree on it).
__device__ __forceinline__ int kmajor64_offset(int r, int kc) {
  return r * 64 + ((kc ^ ((r >> 1) & 3)) << 4);
}

// Byte offset of 16-byte chunk c (k = 8*c..8*c+7) of row r in a K-major tile
// of 16 bfloat16 per row (32 bytes) with the 32-byte swizzle: address bit 4
// is flipped by bit 7 (row bit 2), the layout the tcgen05 descriptor's
// 32-byte swizzle mode reads.
__device__ __forceinline__ int kmajor32_offset(int r, int c) {
  return r * 32 + ((c ^ ((r >> 2) & 1)) << 4);
}

}  // namespace rrb
