// Pieces shared by the two 3xTF32 sgemm kernels (sgemm_tf32x3.cu: operands
// split by a separate pass; sgemm_fused.cu: split inside the MMA kernel): the
// TF32 split itself, the persistent schedule (tiles, k-segments, units,
// rasterization), the split-K plan, and the epilogue warps' barriers.
#pragma once

#include <stdint.h>

#include "tcgen05.cuh"

namespace wg3 {

constexpr int BM = 128;      // UMMA M (cta_group::1), TMEM lanes
constexpr int EPI_WARPS = 4;
constexpr long long WAIT_BUDGET = 4000000000LL;  // SM clocks (~2 s) before a wait gives up
constexpr int GROUP_M = 16;  // tile rows per rasterization group
constexpr int MAX_SEG = 16;  // most k-segments one tile is split into
constexpr int UQ = 4;        // depth of the queue that hands units from the producer to the other roles

#ifdef __CUDACC__
// Round to nearest TF32 (10 explicit mantissa bits), ties away from zero, on
// the bit pattern of a finite float: add half of the dropped 13-bit field and
// truncate. Magnitudes here stay far below the overflow boundary.
__device__ __forceinline__ float rna_tf32(float x) {
  uint32_t u = __float_as_uint(x);
  return __uint_as_float((u + 0x1000u) & 0xFFFFE000u);
}

// An operand the split represents to ~2^-22 relative accuracy with normal
// lo parts: zero, or a finite value with 2^-50 <= |x| <= 2^50.
__device__ __forceinline__ bool split_ok(float x) {
  const float ax = fabsf(x);
  return x == 0.0f || (ax >= 0x1p-50f && ax <= 0x1p50f);
}

// Tile t -> (tile row, tile column), GROUP_M tile rows at a time. Args holds
// tiles_m, tiles_n.
template <class Args>
__device__ __forceinline__ void raster(const Args &a, int t, int &tm, int &tn) {
  const int per_group = GROUP_M * a.tiles_n;
  const int g = t / per_group, first = g * GROUP_M;
  const int rows = a.tiles_m - first < GROUP_M ? a.tiles_m - first : GROUP_M;
  const int r = t % per_group;
  tm = first + r % rows;
  tn = r / rows;
}

// One unit of work: k-blocks [kb0, kb1) of tile t; for a split tile, its
// segment `seg` of sk_split (tile index within the split region: t - dp_tiles).
struct Unit {
  int t, kb0, kb1, seg;
};

// Units are numbered whole tiles first (0 .. dp_tiles-1, in raster order), then
// the split units: unit dp_tiles + v is segment v / sk_tiles of split tile
// v % sk_tiles, so units handed out together cover neighbouring tiles over the
// same k range.
template <class Args>
__device__ __forceinline__ Unit decode(const Args &a, int u) {
  Unit x;
  if (u < a.dp_tiles) {
    x.t = u;
    x.kb0 = 0;
    x.kb1 = a.kt;
    x.seg = -1;
    return x;
  }
  const int v = u - a.dp_tiles;
  x.seg = v / a.sk_tiles;
  x.t = a.dp_tiles + v % a.sk_tiles;
  x.kb0 = (int)((int64_t)a.kt * x.seg / a.sk_split);
  x.kb1 = (int)((int64_t)a.kt * (x.seg + 1) / a.sk_split);
  return x;
}

// Named barrier 1 joins the 128 epilogue threads.
__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
// True on every thread of the COUNT-thread group at named barrier ID iff `v` is
// true on all of them, so a decision to stop is the same for all of its warps
// and no warp is left waiting at a later barrier of the group.
template <int ID, int COUNT = 128>
__device__ __forceinline__ bool group_all(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)v), "n"(ID), "n"(COUNT)
      : "memory");
  return r != 0;
}
// The same with OR.
template <int ID, int COUNT = 128>
__device__ __forceinline__ bool group_any(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)v), "n"(ID), "n"(COUNT)
      : "memory");
  return r != 0;
}
__device__ __forceinline__ bool epi_all(bool v) { return group_all<2>(v); }

// The fp32 alpha/beta epilogue of one thread's row over W consecutive columns
// of C (src/shaders/sgemm_large.wgsl:299-304): C = (alpha == 0 ? 0 : alpha*acc),
// plus beta*C when beta != 0 (C is not read otherwise). Columns at or past n,
// and for gemmtr those outside the triangle, are neither read nor written. When
// all W columns are inside (every chunk but a ragged or diagonal one), the loads
// and stores are straight-line code, so the W old values are in flight
// together: with a per-element test in front of each load the loads went out
// one after another and a 128 x 256 tile's epilogue took 47 us instead of 14.
template <int W>
__device__ __forceinline__ void store_c_row(float *C, int64_t ldc, int64_t row, int64_t col0, int64_t n, int uplo,
                                            float alpha, float beta, const float (&acc)[W]) {
  const bool inside = col0 + W <= n && (uplo == WG_UPLO_FULL || (uplo == WG_UPLO_LOWER ? col0 + W - 1 <= row
                                                                                            : col0 >= row));
  if (inside) {
    float *cp = C + row + col0 * ldc;
    float old[W];
    if (beta != 0.0f) {
#pragma unroll
      for (int j = 0; j < W; j++) old[j] = __ldcg(cp + (int64_t)j * ldc);
    }
#pragma unroll
    for (int j = 0; j < W; j++) {
      const float s = (alpha == 0.0f) ? 0.0f : __fmul_rn(alpha, acc[j]);
      cp[(int64_t)j * ldc] = (beta != 0.0f) ? __fmaf_rn(beta, old[j], s) : s;
    }
    return;
  }
  float old[W];
  if (beta != 0.0f) {
#pragma unroll
    for (int j = 0; j < W; j++) {
      const int64_t col = col0 + j;
      old[j] = col < n && wg_in_triangle(uplo, row, col) ? C[row + col * ldc] : 0.0f;
    }
  }
#pragma unroll
  for (int j = 0; j < W; j++) {
    const int64_t col = col0 + j;
    if (col < n && wg_in_triangle(uplo, row, col)) {
      const float s = (alpha == 0.0f) ? 0.0f : __fmul_rn(alpha, acc[j]);
      C[row + col * ldc] = (beta != 0.0f) ? __fmaf_rn(beta, old[j], s) : s;
    }
  }
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(wgtc::smem_addr(bar)) : "memory");
}
#endif

// ---- host: how a product's tiles are spread over a persistent grid ----

struct Plan {
  int grid;      // CTAs (at most one per SM)
  int dp_tiles;  // tiles taken whole
  int sk_tiles;  // tiles split into sk_split k-segments
  int sk_split;
};

// Whole tiles for every full wave; the rem = T mod G leftover tiles are split
// into s k-segments when that shortens the last wave. In units of one k-block's
// MMA time (about 0.5 us on B200 for a 128 x 256 tile), the last wave costs
// ceil(s*rem/G) rounds of kt/s k-blocks, plus the split's overhead:
// partial-tile writes, the finishing segment's reads of the other s-1 partial
// tiles at the end of the wave, and the round imbalance, about (s-1)*c + 8.
// Measured on B200, c is about 28 for deep tiles (kt = 1024: 128 tiles over 148
// SMs ran fastest whole) and about 4 for shallow ones (kt <= 64: 512^3 and
// 1024^3 ran fastest in 4 segments), so c steps from 4 to 28 at kt = 512. s (at
// most kt/4 and MAX_SEG) minimises the total, and s = 1 keeps the tiles whole.
inline double split_overhead(int kt, int s) { return (kt >= 512 ? 28.0 : 4.0) * (s - 1) + 8.0; }

inline Plan plan_tiles(int G, int tiles_m, int tiles_n, int kt, bool allow_split) {
  const int T = tiles_m * tiles_n;
  Plan p;
  p.grid = T < G ? T : G;
  p.dp_tiles = T;
  p.sk_tiles = 0;
  p.sk_split = 1;
  const int rem = T % G;
  if (!allow_split || rem == 0) return p;
  const int smax = kt / 4 < MAX_SEG ? kt / 4 : MAX_SEG;
  int best_s = 1;
  double best = (double)kt;
  for (int s = 2; s <= smax; s++) {
    const double cost = (double)((s * rem + G - 1) / G) * ((double)kt / s) + split_overhead(kt, s);
    if (cost < best - 1e-9) {
      best = cost;
      best_s = s;
    }
  }
  if (best_s == 1) return p;
  p.dp_tiles = T - rem;
  p.sk_tiles = rem;
  p.sk_split = best_s;
  const int units = rem * best_s;
  p.grid = T - rem >= G ? G : (units < G ? units : G);
  return p;
}

}  // namespace wg3
