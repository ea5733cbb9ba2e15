// 3xTF32 sgemm in one persistent tcgen05 kernel that splits its own operands.
//
// Same arithmetic as sgemm_tf32x3.cu (each fp32 operand x as hi = rna_tf32(x),
// lo = rna_tf32(x - hi); A*B ~= A_lo*B_hi + A_hi*B_lo + A_hi*B_hi accumulated
// in fp32 in TMEM; the reference's alpha/beta epilogue,
// src/shaders/sgemm_large.wgsl:299-304), but the split happens inside the MMA
// kernel instead of in a separate pass over HBM: op(A) and op(B) are read once,
// straight from the caller's matrices, and no split operands are written.
//
// Roles of the 448 threads (one CTA per SM, persistent over 128 x BN tiles):
//  warp 0     TMA producer: takes units (a whole tile, or one k-segment of a
//             split tile) from a work counter, hands each to the other roles
//             through a shared-memory queue, and streams the fp32 k-slices
//             (128 x 16 of op(A), BN x 16 of op(B)) into an SR-deep raw ring.
//             K-contiguous operands arrive in the 64-byte-swizzled K-major
//             layout the tensor core reads; M/N-contiguous ones as plain
//             [16][rows] slices.
//  warps 6-13 split: read each raw slice, write its hi and lo parts into an
//             SC-deep ring of K-major swizzled operand tiles (transposing the
//             M/N-contiguous ones on the way), and note whether any element is
//             outside the split's exact range (non-finite, or |x| outside
//             [2^-50, 2^50]).
//  warp 1     MMA issuer: three tcgen05.mma.kind::tf32 (M=128, N=BN, K=8) per
//             8-wide k step into one of two TMEM accumulators.
//  warps 2-5  epilogue: tcgen05.ld of the other accumulator, 16 columns at a
//             time, and the fp32 alpha/beta store of C (or the partial sums of
//             a split tile; the last segment to arrive adds all segments in k
//             order), overlapping the next unit's MMAs.
// Tile widths BN = 256, 128 or 64 (narrower tiles give small products more
// CTAs); the last wave's tiles can be cut into k-segments as in the other
// kernel. gemmtr calls skip tiles with no element in the triangle.
//
// IEEE semantics: a tile whose operands include an element outside the
// split's exact range is computed on the FFMA pipe instead, by the epilogue
// warps of the CTA that finishes it (ffma_tile_row: the FFMA kernel's
// arithmetic, so its bits) from the untouched C. The CTA-pair form leaves such
// a tile unwritten, gives its entry in a per-tile flag array the call's epoch
// (and the device's fallback word too), and the FFMA kernel launched after it,
// gated on those words, computes exactly the flagged tiles. Every wait is
// clock-bounded (a stalled pipeline sets a bit in the device error word, the
// roles drain, TMEM is freed).
#include <cuda.h>

#include "internal.h"
#include "simt_tile.cuh"
#include "tcgen05.cuh"
#include "tf32x3_common.cuh"

namespace {

using wg3::BM;
using wg3::UQ;
using wg3::WAIT_BUDGET;

constexpr int XF_WARPS = 8;                      // split warps (6 .. 6 + XF_WARPS - 1)
constexpr int XF_THREADS = 32 * XF_WARPS;
constexpr int F_THREADS = 32 * (6 + XF_WARPS);
constexpr int BADQ = 8;  // slots of the per-unit "operands ruled out" word, indexed by unit order
constexpr int EC = 16;   // epilogue columns per TMEM load
constexpr int FG = 2;    // other segments' partial sums loaded together when a split tile is finished

template <int BN_>
struct FS {
  static constexpr int BN = BN_, BK = 16;
  static constexpr int A_TILE = BM * BK * 4, B_TILE = BN * BK * 4;
  static constexpr int RAW = A_TILE + B_TILE, COMP = 2 * RAW;
  static constexpr int SR = BN == 256 ? 3 : (BN == 128 ? 4 : 6);
  static constexpr int SC = BN == 256 ? 3 : (BN == 128 ? 3 : 4);
  static constexpr int TMEM_COLS = BN;  // per accumulator; two of them
  static constexpr size_t SMEM = 1024 + (size_t)SR * RAW + (size_t)SC * COMP + 1024;
  static_assert(B_TILE % 1024 == 0, "tiles keep 1024-byte alignment");
  static_assert(SMEM <= 227 * 1024, "shared memory per CTA");
};

struct FArgs {
  int64_t m, n, k;
  float alpha, beta;
  float *C;
  int64_t ldc;
  unsigned *dwords;      // WG_DW_ERROR (wait timeouts), WG_DW_FALLBACK (any tile ruled out)
  int tiles_m, tiles_n, kt;
  int dp_tiles, sk_tiles, sk_split;
  float *partials;       // split tiles: [sk_tiles * sk_split][BN][BM]
  unsigned *next_unit;   // work counter (zero at launch)
  unsigned *counters;    // split tiles: arrivals (zero at launch, reset by the finishing segment)
  unsigned *tile_bad;    // split tiles: a segment saw ruled-out operands (zero at launch)
  unsigned *tile_flags;  // CTA-pair form: [tiles]: `epoch` where the FFMA kernel computes the tile
  uint32_t epoch;
  int units;
  int uplo;
  // The caller's operands, for tiles computed on the FFMA pipe (one-CTA form).
  const float *A, *B;
  int64_t lda, ldb;
};

// Row i of the C tile at column n0, bn wide, on the FFMA pipe: each element one
// sequential fused multiply-add chain over p = 0..k-1 and then the SIMT GEMM's
// epilogue, so the bits are the FFMA kernel's (and the oracle's). Used for a tile
// whose operands the split ruled out; one thread per row, op(A) loads coalesced
// across the rows, op(B) loads the same address across the warp.
template <int A_K, int B_K>
__device__ __forceinline__ void ffma_tile_row(const FArgs &a, int64_t i, int64_t n0, int bn) {
  constexpr int J = 4;
  const int64_t kk = a.alpha == 0.0f ? 0 : a.k;
  for (int c = 0; c < bn && n0 + c < a.n; c += J) {
    const int64_t j0 = n0 + c;
    float acc[J];
#pragma unroll
    for (int j = 0; j < J; j++) acc[j] = 0.0f;
    for (int64_t p = 0; p < kk; p++) {
      const float av = A_K ? a.A[p + i * a.lda] : a.A[i + p * a.lda];
#pragma unroll
      for (int j = 0; j < J; j++) {
        const int64_t jj = j0 + j;
        const float bv = jj < a.n ? (B_K ? a.B[p + jj * a.ldb] : a.B[jj + p * a.ldb]) : 0.0f;
        acc[j] = __fmaf_rn(av, bv, acc[j]);
      }
    }
#pragma unroll
    for (int j = 0; j < J; j++) {
      const int64_t jj = j0 + j;
      if (jj < a.n && wg_in_triangle(a.uplo, i, jj)) {
        float *cp = a.C + i + jj * a.ldc;
        const float old = a.beta != 0.0f ? *cp : 0.0f;
        *cp = wgsimt::epilogue(acc[j], a.alpha, a.beta, old);
      }
    }
  }
}

// True when x is outside the split's exact range (wg3::split_ok, on the bits:
// |x| as an integer is 0, or within [2^-50, 2^50]; NaN and Inf are above).
__device__ __forceinline__ bool ruled_out(float x) {
  const uint32_t a = __float_as_uint(x) & 0x7FFFFFFFu;
  return (a != 0u) & (a - 0x26800000u > 0x32000000u);
}

__device__ __forceinline__ void split4(const float4 x, float4 &h, float4 &l, bool &bad) {
  bad |= ruled_out(x.x) | ruled_out(x.y) | ruled_out(x.z) | ruled_out(x.w);
  h.x = wg3::rna_tf32(x.x);
  h.y = wg3::rna_tf32(x.y);
  h.z = wg3::rna_tf32(x.z);
  h.w = wg3::rna_tf32(x.w);
  l.x = wg3::rna_tf32(x.x - h.x);
  l.y = wg3::rna_tf32(x.y - h.y);
  l.z = wg3::rna_tf32(x.z - h.z);
  l.w = wg3::rna_tf32(x.w - h.w);
}

// Splits one raw k-slice of ROWS rows into hi and lo K-major tiles (rows of 64
// bytes, 16-byte chunk c of row r at chunk position c ^ ((r >> 1) & 3): the
// 64-byte swizzle TMA writes and the MMA descriptors describe). KMAJ: the raw
// slice is already in that layout, so chunk o maps to chunk o. Otherwise it is
// [16 k][ROWS]: four k values of one row are gathered (a warp reads 32
// consecutive rows per k: conflict-free) and written as one chunk.
template <int ROWS, bool KMAJ>
__device__ __forceinline__ bool split_slice(const uint8_t *raw, uint8_t *hi, uint8_t *lo, int xt) {
  constexpr int STEP = XF_THREADS;
  bool bad = false;
  if (KMAJ) {
    const float4 *src = reinterpret_cast<const float4 *>(raw);
#pragma unroll
    for (int i = xt; i < ROWS * 4; i += STEP) {
      float4 h, l;
      split4(src[i], h, l, bad);
      reinterpret_cast<float4 *>(hi)[i] = h;
      reinterpret_cast<float4 *>(lo)[i] = l;
    }
  } else {
    const float *src = reinterpret_cast<const float *>(raw);
#pragma unroll
    for (int i = xt; i < ROWS * 4; i += STEP) {
      const int r = i % ROWS, c = i / ROWS;
      const float4 x = make_float4(src[(4 * c) * ROWS + r], src[(4 * c + 1) * ROWS + r], src[(4 * c + 2) * ROWS + r],
                                   src[(4 * c + 3) * ROWS + r]);
      float4 h, l;
      split4(x, h, l, bad);
      const int off = r * 64 + ((c ^ ((r >> 1) & 3)) << 4);
      *reinterpret_cast<float4 *>(hi + off) = h;
      *reinterpret_cast<float4 *>(lo + off) = l;
    }
  }
  return bad;
}

// The same split in two phases, so that the split warps can load the raw values
// of two k-slices before any of their stores (loads in flight together): this
// thread's share of one slice of ROWS rows is T = ROWS * 4 / XF_THREADS
// 16-byte chunks.
template <int ROWS>
struct SliceShare {
  static constexpr int T = ROWS * 4 / XF_THREADS;
  float4 x[T];
};

template <int ROWS, bool KMAJ>
__device__ __forceinline__ void slice_load(const uint8_t *raw, int xt, SliceShare<ROWS> &sh) {
#pragma unroll
  for (int t = 0; t < SliceShare<ROWS>::T; t++) {
    const int i = xt + t * XF_THREADS;
    if (KMAJ) {
      sh.x[t] = reinterpret_cast<const float4 *>(raw)[i];
    } else {
      const float *src = reinterpret_cast<const float *>(raw);
      const int r = i % ROWS, c = i / ROWS;
      sh.x[t] = make_float4(src[(4 * c) * ROWS + r], src[(4 * c + 1) * ROWS + r], src[(4 * c + 2) * ROWS + r],
                            src[(4 * c + 3) * ROWS + r]);
    }
  }
}

template <int ROWS, bool KMAJ>
__device__ __forceinline__ bool slice_store(const SliceShare<ROWS> &sh, uint8_t *hi, uint8_t *lo, int xt) {
  bool bad = false;
#pragma unroll
  for (int t = 0; t < SliceShare<ROWS>::T; t++) {
    const int i = xt + t * XF_THREADS;
    float4 h, l;
    split4(sh.x[t], h, l, bad);
    const int off = KMAJ ? i * 16 : (i % ROWS) * 64 + (((i / ROWS) ^ (((i % ROWS) >> 1) & 3)) << 4);
    *reinterpret_cast<float4 *>(hi + off) = h;
    *reinterpret_cast<float4 *>(lo + off) = l;
  }
  return bad;
}

template <class S, int A_K, int B_K>
__global__ void __launch_bounds__(F_THREADS, 1)
tf32x3_fused(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
             const FArgs args) {
  constexpr int BN = S::BN, BK = S::BK, SR = S::SR, SC = S::SC;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t base = wgtc::smem_addr(smem_raw);
  uint8_t *smem = smem_raw + ((1024 - (base & 1023)) & 1023);
  uint8_t *raw = smem;                         // SR x RAW
  uint8_t *comp = smem + (size_t)SR * S::RAW;  // SC x COMP: A_hi, A_lo, B_hi, B_lo
  uint64_t *raw_full = reinterpret_cast<uint64_t *>(comp + (size_t)SC * S::COMP);
  uint64_t *raw_empty = raw_full + SR;
  uint64_t *comp_full = raw_empty + SR;
  uint64_t *comp_empty = comp_full + SC;
  uint64_t *acc_full = comp_empty + SC;  // [2]
  uint64_t *acc_empty = acc_full + 2;    // [2]
  uint64_t *uq_full = acc_empty + 2;     // [UQ]
  uint64_t *uq_empty = uq_full + UQ;     // [UQ]: MMA issuer, epilogue and split have read the slot
  uint64_t *unit_done = uq_empty + UQ;   // [BADQ]: the split has seen all of unit n's operands
  volatile int *uq = reinterpret_cast<volatile int *>(unit_done + BADQ);
  volatile int *unit_bad = uq + UQ;      // [BADQ]
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(const_cast<int *>(unit_bad) + BADQ);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
  volatile unsigned *last_flag = reinterpret_cast<volatile unsigned *>(tmem_slot + 2);
  volatile unsigned *seg_bad = reinterpret_cast<volatile unsigned *>(tmem_slot + 3);
  wg_pdl_trigger();  // the gated FFMA launch after this one may be scheduled early; it waits for this kernel

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < SR; s++) {
      wgtc::mbar_init(&raw_full[s], 1);
      wgtc::mbar_init(&raw_empty[s], XF_WARPS);
    }
    for (int s = 0; s < SC; s++) {
      wgtc::mbar_init(&comp_full[s], XF_WARPS);
      wgtc::mbar_init(&comp_empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      wgtc::mbar_init(&acc_full[b], 1);
      wgtc::mbar_init(&acc_empty[b], 32 * wg3::EPI_WARPS);
    }
    for (int i = 0; i < UQ; i++) {
      wgtc::mbar_init(&uq_full[i], 1);
      wgtc::mbar_init(&uq_empty[i], 2 + XF_WARPS);  // MMA issuer, epilogue, each split warp
    }
    for (int i = 0; i < BADQ; i++) {
      wgtc::mbar_init(&unit_done[i], XF_WARPS);
      unit_bad[i] = 0;
    }
    *abort_flag = 0;
    wgtc::fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    wgtc::prefetch_tensormap(&map_a);
    wgtc::prefetch_tensormap(&map_b);
  }
  if (warp == 1) {
    wgtc::tmem_alloc(tmem_slot, 2 * S::TMEM_COLS);
    wgtc::tmem_relinquish();
  }
  wgtc::tc_fence_before();
  __syncthreads();
  wgtc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---- TMA producer ----
      int64_t g = 0;
      bool ok = true;
      for (int n = 0; ok; n++) {
        const int slot = n % UQ;
        int un = n == 0 ? (int)blockIdx.x : (int)gridDim.x + (int)atomicAdd(args.next_unit, 1u);
        while (args.uplo != WG_UPLO_FULL && un < args.units) {
          int tm0, tn0;
          wg3::raster(args, wg3::decode(args, un).t, tm0, tn0);
          if (!wg_tile_outside(args.uplo, (int64_t)tm0 * BM, BM, (int64_t)tn0 * BN, BN)) break;
          un = (int)gridDim.x + (int)atomicAdd(args.next_unit, 1u);
        }
        if (un >= args.units) un = -1;  // no work left: tells the other roles to stop
        if (!wgtc::mbar_wait_bounded(&uq_empty[slot], ((uint32_t)(n / UQ) & 1u) ^ 1u, WAIT_BUDGET) ||
            *abort_flag) {
          atomicOr(args.dwords + WG_DW_ERROR, WG_DERR_TMA_WAIT);
          *abort_flag = 1;
          break;
        }
        uq[slot] = un;
        wg3::mbar_arrive(&uq_full[slot]);
        if (un < 0) break;
        const wg3::Unit u = wg3::decode(args, un);
        int tm, tn;
        wg3::raster(args, u.t, tm, tn);
        for (int kb = u.kb0; kb < u.kb1; kb++, g++) {
          const int s = (int)(g % SR);
          const uint32_t ph = (uint32_t)(g / SR) & 1u;
          if (!wgtc::mbar_wait_bounded(&raw_empty[s], ph ^ 1u, WAIT_BUDGET) || *abort_flag) {
            atomicOr(args.dwords + WG_DW_ERROR, WG_DERR_TMA_WAIT);
            *abort_flag = 1;
            ok = false;
            break;
          }
          uint8_t *st = raw + (size_t)s * S::RAW;
          wgtc::mbar_arrive_expect_tx(&raw_full[s], S::RAW);
          const int kc = kb * BK;
          if (A_K)
            wgtc::tma_load_2d(st, &map_a, &raw_full[s], kc, tm * BM);
          else
            wgtc::tma_load_2d(st, &map_a, &raw_full[s], tm * BM, kc);
          if (B_K)
            wgtc::tma_load_2d(st + S::A_TILE, &map_b, &raw_full[s], kc, tn * BN);
          else
            wgtc::tma_load_2d(st + S::A_TILE, &map_b, &raw_full[s], tn * BN, kc);
        }
      }
      // Every copy issued lands before the CTA can exit.
      for (int64_t q = g - SR > 0 ? g - SR : 0; q < g; q++)
        wgtc::mbar_wait_bounded(&raw_full[q % SR], (uint32_t)(q / SR) & 1u, WAIT_BUDGET);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---- MMA issuer ----
      constexpr uint32_t idesc = wgtc::idesc_tf32(BM, BN);
      int64_t h = 0;
      bool ok = true;
      for (int n = 0; ok; n++) {
        const int slot = n % UQ;
        if (!wgtc::mbar_wait_bounded(&uq_full[slot], (uint32_t)(n / UQ) & 1u, WAIT_BUDGET) || *abort_flag) {
          atomicOr(args.dwords + WG_DW_ERROR, WG_DERR_MMA_WAIT);
          *abort_flag = 1;
          break;
        }
        const int un = uq[slot];
        wg3::mbar_arrive(&uq_empty[slot]);
        if (un < 0) break;
        const wg3::Unit u = wg3::decode(args, un);
        const int b = n & 1;
        const uint32_t use = (uint32_t)(n >> 1);
        if (!wgtc::mbar_wait_bounded(&acc_empty[b], (use & 1u) ^ 1u, WAIT_BUDGET) || *abort_flag) {
          atomicOr(args.dwords + WG_DW_ERROR, WG_DERR_MMA_WAIT);
          *abort_flag = 1;
          break;
        }
        wgtc::tc_fence_after();
        const uint32_t d_tmem = tmem + (uint32_t)(b * S::TMEM_COLS);
        for (int kb = u.kb0; kb < u.kb1; kb++, h++) {
          const int c = (int)(h % SC);
          if (!wgtc::mbar_wait_bounded(&comp_full[c], (uint32_t)(h / SC) & 1u, WAIT_BUDGET) || *abort_flag) {
            atomicOr(args.dwords + WG_DW_ERROR, WG_DERR_MMA_WAIT);
            *abort_flag = 1;
            ok = false;
            break;
          }
          wgtc::tc_fence_after();
          const uint32_t st = wgtc::smem_addr(comp + (size_t)c * S::COMP);
          const uint32_t a_hi = st, a_lo = st + S::A_TILE, b_hi = st + 2 * S::A_TILE, b_lo = b_hi + S::B_TILE;
#pragma unroll
          for (int kk = 0; kk < BK / 8; kk++) {
            const uint32_t off = kk * 32;  // 8 tf32 = 32 bytes along K inside the 64-byte rows
            const uint64_t dah = wgtc::smem_desc_kmajor(a_hi + off, 64);
            const uint64_t dal = wgtc::smem_desc_kmajor(a_lo + off, 64);
            const uint64_t dbh = wgtc::smem_desc_kmajor(b_hi + off, 64);
            const uint64_t dbl = wgtc::smem_desc_kmajor(b_lo + off, 64);
            const uint32_t acc0 = (kb > u.kb0 || kk > 0) ? 1u : 0u;
            wgtc::mma_tf32(d_tmem, dal, dbh, idesc, acc0);  // small terms first
            wgtc::mma_tf32(d_tmem, dah, dbl, idesc, 1u);
            wgtc::mma_tf32(d_tmem, dah, dbh, idesc, 1u);
          }
          wgtc::mma_commit(&comp_empty[c]);  // frees the operand stage once these MMAs have read it
        }
        wgtc::mma_commit(&acc_full[b]);
      }
    }
  } else if (warp >= 6) {
    // ---- split: raw fp32 slices -> hi / lo operand tiles. Each warp works on
    // its share of every slice and signals on its own (the barriers count the
    // warps), so no warp waits for another. ----
    const int xt = threadIdx.x - 192;
    int64_t g = 0, h = 0;
    for (int n = 0;; n++) {
      const int slot = n % UQ;
      const bool got = wgtc::mbar_wait_bounded(&uq_full[slot], (uint32_t)(n / UQ) & 1u, WAIT_BUDGET);
      const int un = got ? uq[slot] : -1;
      if (!__all_sync(0xffffffffu, got && *abort_flag == 0)) {
        if (!got) atomicOr(args.dwords + WG_DW_ERROR, WG_DERR_TMA_WAIT);
        *abort_flag = 1;
        break;
      }
      __syncwarp();
      if (lane == 0) wg3::mbar_arrive(&uq_empty[slot]);
      if (un < 0) break;
      const wg3::Unit u = wg3::decode(args, un);
      bool bad = false, failed = false;
      // Two k-slices per step where the unit has them: their raw values are all
      // loaded before any split value is stored, and the fence and the
      // signalling are paid once per pair.
      for (int kb = u.kb0; kb < u.kb1;) {
        const int nk = kb + 1 < u.kb1 ? 2 : 1;
        const int s0 = (int)(g % SR), c0 = (int)(h % SC);
        const int s1 = (int)((g + 1) % SR), c1 = (int)((h + 1) % SC);
        bool ok = wgtc::mbar_wait_bounded(&raw_full[s0], (uint32_t)(g / SR) & 1u, WAIT_BUDGET) &&
                  wgtc::mbar_wait_bounded(&comp_empty[c0], ((uint32_t)(h / SC) & 1u) ^ 1u, WAIT_BUDGET);
        if (ok && nk == 2)
          ok = wgtc::mbar_wait_bounded(&raw_full[s1], (uint32_t)((g + 1) / SR) & 1u, WAIT_BUDGET) &&
               wgtc::mbar_wait_bounded(&comp_empty[c1], ((uint32_t)((h + 1) / SC) & 1u) ^ 1u, WAIT_BUDGET);
        if (!__all_sync(0xffffffffu, ok && *abort_flag == 0)) {
          if (!ok) atomicOr(args.dwords + WG_DW_ERROR, WG_DERR_TMA_WAIT);
          *abort_flag = 1;
          failed = true;
          break;
        }
        const uint8_t *rs0 = raw + (size_t)s0 * S::RAW, *rs1 = raw + (size_t)s1 * S::RAW;
        uint8_t *cs0 = comp + (size_t)c0 * S::COMP, *cs1 = comp + (size_t)c1 * S::COMP;
        SliceShare<BM> a0, a1;
        SliceShare<BN> b0, b1;
        slice_load<BM, A_K != 0>(rs0, xt, a0);
        slice_load<BN, B_K != 0>(rs0 + S::A_TILE, xt, b0);
        if (nk == 2) {
          slice_load<BM, A_K != 0>(rs1, xt, a1);
          slice_load<BN, B_K != 0>(rs1 + S::A_TILE, xt, b1);
        }
        bad |= slice_store<BM, A_K != 0>(a0, cs0, cs0 + S::A_TILE, xt);
        bad |= slice_store<BN, B_K != 0>(b0, cs0 + 2 * S::A_TILE, cs0 + 2 * S::A_TILE + S::B_TILE, xt);
        if (nk == 2) {
          bad |= slice_store<BM, A_K != 0>(a1, cs1, cs1 + S::A_TILE, xt);
          bad |= slice_store<BN, B_K != 0>(b1, cs1 + 2 * S::A_TILE, cs1 + 2 * S::A_TILE + S::B_TILE, xt);
        }
        wgtc::fence_proxy_async_smem();  // the MMAs read these tiles through the async proxy
        __syncwarp();
        if (lane == 0) {
          wg3::mbar_arrive(&comp_full[c0]);
          wg3::mbar_arrive(&raw_empty[s0]);
          if (nk == 2) {
            wg3::mbar_arrive(&comp_full[c1]);
            wg3::mbar_arrive(&raw_empty[s1]);
          }
        }
        kb += nk;
        g += nk;
        h += nk;
      }
      if (failed) break;
      if (__any_sync(0xffffffffu, bad) && lane == 0) atomicOr(const_cast<int *>(&unit_bad[n % BADQ]), 1);
      __syncwarp();
      if (lane == 0) wg3::mbar_arrive(&unit_done[n % BADQ]);
    }
  } else {
    // ---- epilogue: TMEM -> registers -> C (or a partial-sum slot) ----
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int row_in_tile = q * 32 + lane;
    const float alpha = args.alpha, beta = args.beta;
    for (int n = 0;; n++) {
      const int slot = n % UQ;
      const bool got = wgtc::mbar_wait_bounded(&uq_full[slot], (uint32_t)(n / UQ) & 1u, WAIT_BUDGET);
      const int un = got ? uq[slot] : -1;
      if (!wg3::epi_all(got && *abort_flag == 0)) {
        if (!got) atomicOr(args.dwords + WG_DW_ERROR, WG_DERR_MMA_WAIT);
        *abort_flag = 1;
        break;
      }
      if (threadIdx.x == 64) wg3::mbar_arrive(&uq_empty[slot]);
      if (un < 0) break;
      const wg3::Unit u = wg3::decode(args, un);
      const int b = n & 1;
      const uint32_t use = (uint32_t)(n >> 1);
      const bool ready = wgtc::mbar_wait_bounded(&acc_full[b], use & 1u, WAIT_BUDGET) &&
                         wgtc::mbar_wait_bounded(&unit_done[n % BADQ], (uint32_t)(n / BADQ) & 1u, WAIT_BUDGET);
      if (!wg3::epi_all(ready && *abort_flag == 0)) {
        if (!ready) atomicOr(args.dwords + WG_DW_ERROR, WG_DERR_MMA_WAIT);
        *abort_flag = 1;
        break;
      }
      wgtc::tc_fence_after();
      const bool bad = unit_bad[n % BADQ] != 0;
      wg3::epi_bar();  // every thread has read the word before it is cleared for unit n + BADQ
      if (threadIdx.x == 64) unit_bad[n % BADQ] = 0;
      int tm, tn;
      wg3::raster(args, u.t, tm, tn);
      const int64_t row = (int64_t)tm * BM + row_in_tile;
      const int64_t n0 = (int64_t)tn * BN;
      const uint32_t trow = tmem + (uint32_t)(b * S::TMEM_COLS) + ((uint32_t)(q * 32) << 16);
      const bool whole = u.seg < 0;
      bool finish = whole, ruled_out = bad;
      const int local = u.t - args.dp_tiles;
      if (!whole) {
        // Leave this segment's partial sums (unless its operands were ruled out),
        // then count arrivals on the tile.
        if (!bad) {
          float *part = args.partials + ((int64_t)local * args.sk_split + u.seg) * BN * BM + row_in_tile;
          for (int c = 0; c < BN; c += EC) {
            uint32_t r[EC];
            wgtc::tmem_ld_32x32b_x16(trow + (uint32_t)c, r);
            wgtc::tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < EC; j++) part[(int64_t)(c + j) * BM] = __uint_as_float(r[j]);
          }
        }
        if (bad && threadIdx.x == 64) atomicOr(args.tile_bad + local, 1u);
        __threadfence();
        wg3::epi_bar();
        if (threadIdx.x == 64) {
          const unsigned prev = atomicAdd(args.counters + local, 1u);
          const bool last = prev == (unsigned)(args.sk_split - 1);
          if (last) {
            args.counters[local] = 0;  // ready for the next call on this workspace
            *seg_bad = atomicExch(args.tile_bad + local, 0u);
          }
          *last_flag = last ? 1u : 0u;
          __threadfence();
        }
        wg3::epi_bar();
        finish = *last_flag != 0;
        if (finish) {
          __threadfence();  // order the reads of the other segments' partial sums
          ruled_out = *seg_bad != 0;
        }
      }
      if (finish && ruled_out) {
        // Operands the split cannot carry: this tile's C on the FFMA pipe, with
        // the reference's IEEE semantics. The call's first such tile counts one
        // fallback.
        if (threadIdx.x == 64 && atomicExch(args.dwords + WG_DW_FALLBACK, args.epoch) != args.epoch)
          atomicAdd(args.dwords + WG_DW_FALLBACKS, 1u);
        if (row < args.m) ffma_tile_row<A_K, B_K>(args, row, n0, BN);
      } else if (finish) {
        const int nseg = whole ? 1 : args.sk_split;
        const int own = whole ? 0 : u.seg;
        const float *part0 = whole ? nullptr : args.partials + (int64_t)local * args.sk_split * BN * BM + row_in_tile;
        const bool in_rows = row < args.m;
        for (int c = 0; c < BN; c += EC) {
          uint32_t r[EC];
          wgtc::tmem_ld_32x32b_x16(trow + (uint32_t)c, r);
          wgtc::tmem_ld_wait();
          float acc[EC];
#pragma unroll
          for (int j = 0; j < EC; j++) acc[j] = __uint_as_float(r[j]);
          if (nseg > 1) {
            // Segments in k order; the partial sums of up to FG other segments
            // are loaded together (one memory round trip per group), this CTA's
            // own comes from TMEM. Group [s, e) holds FG others and, where it
            // falls among them, this CTA's own segment.
            float sum[EC];
            for (int s = 0; s < nseg;) {
              const bool own_near = own >= s && own <= s + FG;
              const int e = s + FG + (own_near ? 1 : 0) < nseg ? s + FG + (own_near ? 1 : 0) : nseg;
              const bool own_in = own >= s && own < e;
              float v[FG][EC];
#pragma unroll
              for (int qq = 0; qq < FG; qq++) {
                const int sgi = s + qq + ((own_in && s + qq >= own) ? 1 : 0);  // the qq-th other segment
                if (sgi < e) {
                  const float *p = part0 + ((int64_t)sgi * BN + c) * BM;
#pragma unroll
                  for (int j = 0; j < EC; j++) v[qq][j] = __ldcg(p + (int64_t)j * BM);
                }
              }
#pragma unroll
              for (int idx = 0; idx <= FG; idx++) {
                const int t = s + idx;
                if (t < e) {
                  const int vi = idx - ((own_in && t > own) ? 1 : 0);
#pragma unroll
                  for (int j = 0; j < EC; j++) {
                    const float x = t == own ? acc[j] : (vi == 0 ? v[0][j] : v[1][j]);
                    sum[j] = t == 0 ? x : sum[j] + x;
                  }
                }
              }
              s = e;
            }
#pragma unroll
            for (int j = 0; j < EC; j++) acc[j] = sum[j];
          }
          if (in_rows) wg3::store_c_row<EC>(args.C, args.ldc, row, n0 + c, args.n, args.uplo, alpha, beta, acc);
        }
      }
      wgtc::tc_fence_before();
      wg3::mbar_arrive(&acc_empty[b]);  // accumulator b may be refilled
    }
  }

  wgtc::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    wgtc::tc_fence_after();
    wgtc::tmem_dealloc(tmem, 2 * S::TMEM_COLS);
  }
}

// ---- the CTA-pair form (cta_group::2) ---------------------------------------
//
// The same split-in-kernel 3xTF32 product over pairs of CTAs on neighbouring
// SMs (a cluster of two). A pair owns 256 x 256 tiles of C: each CTA loads and
// splits its 128 rows of op(A) and 128 of the tile's 256 rows of op(B), and one
// thread of the first CTA issues tcgen05.mma.cta_group::2 (M = 256, N = 256),
// which reads the A and B halves of both CTAs and leaves each CTA's 128 rows of
// the tile in that CTA's TMEM. Per SM and 16-deep k-block that is 16 KB of TMA
// traffic, 48 KB written by the split and 48 KB read by the MMAs, against 24,
// 48 and 72 KB for a single CTA holding a 128 x 256 tile: the pair fits the
// split inside the shared-memory bandwidth the MMAs leave.
//
// Work is scheduled statically (unit u of the decode order goes to pair
// u mod pairs), so both CTAs walk the same units without a queue between them.
// Synchronisation across the pair: each CTA's split warps arrive on the first
// CTA's operand-ready barrier (remotely from the second CTA); the MMA commits
// multicast to both CTAs' operand-free and accumulator-ready barriers; both
// epilogues arrive on the first CTA's accumulator-free barrier; each split
// announces per unit whether its operands were ruled out to both CTAs. Every
// wait is clock-bounded; both CTAs reach the closing cluster barrier on every
// path.

constexpr int P_BN = 256;                  // tile columns of a pair (128 B rows per CTA)
constexpr int P_HALF = P_BN / 2;
constexpr int P_A = BM * 16 * 4;           // 8 KB: one CTA's k-slice of op(A)
constexpr int P_B = P_HALF * 16 * 4;       // 8 KB: one CTA's k-slice of op(B)
constexpr int P_RAW = P_A + P_B, P_COMP = 2 * P_RAW;
constexpr int P_SR = 4, P_SC = 4;
constexpr size_t P_SMEM = 1024 + (size_t)P_SR * P_RAW + (size_t)P_SC * P_COMP + 1024;
static_assert(P_SMEM <= 227 * 1024, "shared memory per CTA");

template <int A_K, int B_K>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(F_THREADS, 1)
tf32x3_fused_pair(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                  const FArgs args) {
  constexpr int BK = 16, SR = P_SR, SC = P_SC;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t base = wgtc::smem_addr(smem_raw);
  uint8_t *smem = smem_raw + ((1024 - (base & 1023)) & 1023);
  uint8_t *raw = smem;
  uint8_t *comp = smem + (size_t)SR * P_RAW;
  uint64_t *raw_full = reinterpret_cast<uint64_t *>(comp + (size_t)SC * P_COMP);
  uint64_t *raw_empty = raw_full + SR;
  uint64_t *comp_full = raw_empty + SR;   // first CTA: both CTAs' split warps arrive
  uint64_t *comp_empty = comp_full + SC;  // both CTAs: the MMA's multicast commit
  uint64_t *acc_full = comp_empty + SC;   // [2], both CTAs: the MMA's multicast commit
  uint64_t *acc_empty = acc_full + 2;     // [2], first CTA: both CTAs' epilogue threads
  uint64_t *unit_done = acc_empty + 2;    // [BADQ], both CTAs: both splits arrive
  volatile unsigned *unit_bad = reinterpret_cast<volatile unsigned *>(unit_done + BADQ);  // [BADQ]
  uint32_t *tmem_slot = const_cast<uint32_t *>(reinterpret_cast<volatile uint32_t *>(unit_bad + BADQ));
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
  volatile unsigned *last_flag = reinterpret_cast<volatile unsigned *>(tmem_slot + 2);
  volatile unsigned *seg_bad = reinterpret_cast<volatile unsigned *>(tmem_slot + 3);
  wg_pdl_trigger();  // the gated FFMA launch after this one may be scheduled early; it waits for this kernel

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = wgtc::cluster_ctarank();
  const int pair = (int)(blockIdx.x >> 1), pairs = (int)(gridDim.x >> 1);

  if (threadIdx.x == 0) {
    for (int s = 0; s < SR; s++) {
      wgtc::mbar_init(&raw_full[s], 1);
      wgtc::mbar_init(&raw_empty[s], XF_WARPS);
    }
    for (int s = 0; s < SC; s++) {
      wgtc::mbar_init(&comp_full[s], 2 * XF_WARPS);
      wgtc::mbar_init(&comp_empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      wgtc::mbar_init(&acc_full[b], 1);
      wgtc::mbar_init(&acc_empty[b], 2 * 32 * wg3::EPI_WARPS);
    }
    for (int i = 0; i < BADQ; i++) {
      wgtc::mbar_init(&unit_done[i], 2 * XF_WARPS);  // every split warp of both CTAs
      unit_bad[i] = 0;
    }
    *abort_flag = 0;
    wgtc::fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    wgtc::prefetch_tensormap(&map_a);
    wgtc::prefetch_tensormap(&map_b);
  }
  if (warp == 1) {
    wgtc::tmem_alloc_pair(tmem_slot, 2 * P_BN);
    wgtc::tmem_relinquish_pair();
  }
  wgtc::tc_fence_before();
  __syncthreads();
  __syncwarp();
  wgtc::cluster_sync();  // both CTAs' barriers exist before any remote arrival
  wgtc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // The pair's units, in order: u = pair, pair + pairs, ... (gemmtr skips the
  // tiles with no element in the triangle; both CTAs skip the same ones).
  auto next_unit = [&](int u) -> int {
    for (u += pairs; u < args.units; u += pairs) {
      if (args.uplo == WG_UPLO_FULL) return u;
      int tm0, tn0;
      wg3::raster(args, wg3::decode(args, u).t, tm0, tn0);
      if (!wg_tile_outside(args.uplo, (int64_t)tm0 * 2 * BM, 2 * BM, (int64_t)tn0 * P_BN, P_BN)) return u;
    }
    return args.units;
  };
  const int first = next_unit(pair - pairs);

  if (warp == 0) {
    if (lane == 0) {
      // ---- TMA producer: this CTA's halves of each k-slice ----
      int64_t g = 0;
      bool ok = true;
      for (int un = first; ok && un < args.units; un = next_unit(un)) {
        const wg3::Unit u = wg3::decode(args, un);
        int tm, tn;
        wg3::raster(args, u.t, tm, tn);
        const int row_a = tm * 2 * BM + (int)rank * BM, row_b = tn * P_BN + (int)rank * P_HALF;
        for (int kb = u.kb0; kb < u.kb1; kb++, g++) {
          const int s = (int)(g % SR);
          if (!wgtc::mbar_wait_bounded(&raw_empty[s], ((uint32_t)(g / SR) & 1u) ^ 1u, WAIT_BUDGET) || *abort_flag) {
            atomicOr(args.dwords + WG_DW_ERROR, WG_DERR_TMA_WAIT);
            *abort_flag = 1;
            ok = false;
            break;
          }
          uint8_t *st = raw + (size_t)s * P_RAW;
          wgtc::mbar_arrive_expect_tx(&raw_full[s], P_RAW);
          const int kc = kb * BK;
          if (A_K)
            wgtc::tma_load_2d(st, &map_a, &raw_full[s], kc, row_a);
          else
            wgtc::tma_load_2d(st, &map_a, &raw_full[s], row_a, kc);
          if (B_K)
            wgtc::tma_load_2d(st + P_A, &map_b, &raw_full[s], kc, row_b);
          else
            wgtc::tma_load_2d(st + P_A, &map_b, &raw_full[s], row_b, kc);
        }
      }
      for (int64_t q = g - SR > 0 ? g - SR : 0; q < g; q++)
        wgtc::mbar_wait_bounded(&raw_full[q % SR], (uint32_t)(q / SR) & 1u, WAIT_BUDGET);
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // ---- MMA issuer of the pair ----
      constexpr uint32_t idesc = wgtc::idesc_tf32(2 * BM, P_BN);
      int64_t h = 0;
      int it = 0;
      bool ok = true;
      for (int un = first; ok && un < args.units; un = next_unit(un), it++) {
        const wg3::Unit u = wg3::decode(args, un);
        const int b = it & 1;
        const uint32_t use = (uint32_t)(it >> 1);
        if (!wgtc::mbar_wait_bounded_cluster(&acc_empty[b], (use & 1u) ^ 1u, WAIT_BUDGET) || *abort_flag) {
          atomicOr(args.dwords + WG_DW_ERROR, WG_DERR_MMA_WAIT);
          *abort_flag = 1;
          break;
        }
        wgtc::tc_fence_after();
        const uint32_t d_tmem = tmem + (uint32_t)(b * P_BN);
        for (int kb = u.kb0; kb < u.kb1; kb++, h++) {
          const int c = (int)(h % SC);
          if (!wgtc::mbar_wait_bounded_cluster(&comp_full[c], (uint32_t)(h / SC) & 1u, WAIT_BUDGET) ||
              *abort_flag) {
            atomicOr(args.dwords + WG_DW_ERROR, WG_DERR_MMA_WAIT);
            *abort_flag = 1;
            ok = false;
            break;
          }
          wgtc::tc_fence_after();
          const uint32_t st = wgtc::smem_addr(comp + (size_t)c * P_COMP);
          const uint32_t a_hi = st, a_lo = st + P_A, b_hi = st + 2 * P_A, b_lo = b_hi + P_B;
#pragma unroll
          for (int kk = 0; kk < BK / 8; kk++) {
            const uint32_t off = kk * 32;
            const uint64_t dah = wgtc::smem_desc_kmajor(a_hi + off, 64);
            const uint64_t dal = wgtc::smem_desc_kmajor(a_lo + off, 64);
            const uint64_t dbh = wgtc::smem_desc_kmajor(b_hi + off, 64);
            const uint64_t dbl = wgtc::smem_desc_kmajor(b_lo + off, 64);
            const uint32_t acc0 = (kb > u.kb0 || kk > 0) ? 1u : 0u;
            wgtc::mma_tf32_pair(d_tmem, dal, dbh, idesc, acc0);
            wgtc::mma_tf32_pair(d_tmem, dah, dbl, idesc, 1u);
            wgtc::mma_tf32_pair(d_tmem, dah, dbh, idesc, 1u);
          }
          wgtc::mma_commit_pair(&comp_empty[c], 0x3);  // both CTAs may refill stage c
        }
        if (!ok) break;
        wgtc::mma_commit_pair(&acc_full[b], 0x3);  // both CTAs' rows of the tile are complete
      }
    }
  } else if (warp >= 6) {
    // ---- split: this CTA's raw halves -> hi / lo operand tiles (each warp on its
    // own share, signalling on its own) ----
    const int xt = threadIdx.x - 192;
    const uint32_t comp_full_first = wgtc::mapa_shared(wgtc::smem_addr(comp_full), 0);
    const uint32_t peer = rank ^ 1u;
    int64_t g = 0, h = 0;
    int it = 0;
    for (int un = first; un < args.units; un = next_unit(un), it++) {
      const wg3::Unit u = wg3::decode(args, un);
      bool bad = false, failed = false;
      for (int kb = u.kb0; kb < u.kb1; kb++, g++, h++) {
        const int s = (int)(g % SR), c = (int)(h % SC);
        const bool okr = wgtc::mbar_wait_bounded(&raw_full[s], (uint32_t)(g / SR) & 1u, WAIT_BUDGET);
        const bool okc =
            wgtc::mbar_wait_bounded_cluster(&comp_empty[c], ((uint32_t)(h / SC) & 1u) ^ 1u, WAIT_BUDGET);
        if (!__all_sync(0xffffffffu, okr && okc && *abort_flag == 0)) {
          if (!(okr && okc)) atomicOr(args.dwords + WG_DW_ERROR, WG_DERR_TMA_WAIT);
          *abort_flag = 1;
          failed = true;
          break;
        }
        const uint8_t *rs = raw + (size_t)s * P_RAW;
        uint8_t *cs = comp + (size_t)c * P_COMP;
        bad |= split_slice<BM, A_K != 0>(rs, cs, cs + P_A, xt);
        bad |= split_slice<P_HALF, B_K != 0>(rs + P_A, cs + 2 * P_A, cs + 2 * P_A + P_B, xt);
        wgtc::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          wgtc::mbar_arrive_cluster(comp_full_first + (uint32_t)(c * 8));
          wg3::mbar_arrive(&raw_empty[s]);
        }
      }
      if (failed) break;
      const bool any_bad = __any_sync(0xffffffffu, bad);
      if (lane == 0) {
        const int q = it % BADQ;
        if (any_bad) {
          atomicOr(const_cast<unsigned *>(&unit_bad[q]), 1u);
          wgtc::red_or_cluster(wgtc::mapa_shared(wgtc::smem_addr(const_cast<unsigned *>(&unit_bad[q])), peer), 1u);
        }
        wgtc::mbar_arrive_cluster(wgtc::mapa_shared(wgtc::smem_addr(&unit_done[q]), 0));
        wgtc::mbar_arrive_cluster(wgtc::mapa_shared(wgtc::smem_addr(&unit_done[q]), 1));
      }
    }
  } else if (warp >= 2) {
    // ---- epilogue: this CTA's 128 rows of the pair's tile ----
    const int q = warp & 3;
    const int row_in_tile = q * 32 + lane;
    const float alpha = args.alpha, beta = args.beta;
    const uint32_t acc_empty_first = wgtc::mapa_shared(wgtc::smem_addr(acc_empty), 0);
    const int tiles_m128 = 2 * args.tiles_m;
    int it = 0;
    for (int un = first; un < args.units; un = next_unit(un), it++) {
      const wg3::Unit u = wg3::decode(args, un);
      const int b = it & 1;
      const uint32_t use = (uint32_t)(it >> 1);
      const bool ready =
          wgtc::mbar_wait_bounded_cluster(&acc_full[b], use & 1u, WAIT_BUDGET) &&
          wgtc::mbar_wait_bounded_cluster(&unit_done[it % BADQ], (uint32_t)(it / BADQ) & 1u, WAIT_BUDGET);
      if (!wg3::epi_all(ready && *abort_flag == 0)) {
        if (!ready) atomicOr(args.dwords + WG_DW_ERROR, WG_DERR_MMA_WAIT);
        *abort_flag = 1;
        break;
      }
      wgtc::tc_fence_after();
      const bool bad = unit_bad[it % BADQ] != 0;
      wg3::epi_bar();  // every thread has read the word before it is cleared for unit it + BADQ
      if (threadIdx.x == 64) unit_bad[it % BADQ] = 0;
      int tm, tn;
      wg3::raster(args, u.t, tm, tn);
      const int half = tm * 2 + (int)rank;  // this CTA's 128-row block
      const int64_t row = (int64_t)half * BM + row_in_tile;
      const int64_t n0 = (int64_t)tn * P_BN;
      const uint32_t trow = tmem + (uint32_t)(b * P_BN) + ((uint32_t)(q * 32) << 16);
      const bool whole = u.seg < 0;
      bool finish = whole, ruled_out = bad;
      const int local = (u.t - args.dp_tiles) * 2 + (int)rank;  // split tile half
      if (!whole) {
        if (!bad) {
          float *part = args.partials + ((int64_t)local * args.sk_split + u.seg) * P_BN * BM + row_in_tile;
          for (int c = 0; c < P_BN; c += EC) {
            uint32_t r[EC];
            wgtc::tmem_ld_32x32b_x16(trow + (uint32_t)c, r);
            wgtc::tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < EC; j++) part[(int64_t)(c + j) * BM] = __uint_as_float(r[j]);
          }
        }
        if (bad && threadIdx.x == 64) atomicOr(args.tile_bad + local, 1u);
        __threadfence();
        wg3::epi_bar();
        if (threadIdx.x == 64) {
          const unsigned prev = atomicAdd(args.counters + local, 1u);
          const bool last = prev == (unsigned)(args.sk_split - 1);
          if (last) {
            args.counters[local] = 0;
            *seg_bad = atomicExch(args.tile_bad + local, 0u);
          }
          *last_flag = last ? 1u : 0u;
          __threadfence();
        }
        wg3::epi_bar();
        finish = *last_flag != 0;
        if (finish) {
          __threadfence();
          ruled_out = *seg_bad != 0;
        }
      }
      if (finish && ruled_out) {
        if (threadIdx.x == 64) {
          args.tile_flags[half + (int64_t)tn * tiles_m128] = args.epoch;
          atomicExch(args.dwords + WG_DW_FALLBACK, args.epoch);
        }
      } else if (finish) {
        const int nseg = whole ? 1 : args.sk_split;
        const int own = whole ? 0 : u.seg;
        const float *part0 = whole ? nullptr : args.partials + (int64_t)local * args.sk_split * P_BN * BM + row_in_tile;
        const bool in_rows = row < args.m;
        for (int c = 0; c < P_BN; c += EC) {
          uint32_t r[EC];
          wgtc::tmem_ld_32x32b_x16(trow + (uint32_t)c, r);
          wgtc::tmem_ld_wait();
          float acc[EC];
#pragma unroll
          for (int j = 0; j < EC; j++) acc[j] = __uint_as_float(r[j]);
          if (nseg > 1) {
            float sum[EC];
            for (int g0 = 0; g0 < nseg; g0 += 2) {
              float v[2][EC];
#pragma unroll
              for (int qq = 0; qq < 2; qq++) {
                const int sgi = g0 + qq;
                if (sgi < nseg && sgi != own) {
                  const float *p = part0 + ((int64_t)sgi * P_BN + c) * BM;
#pragma unroll
                  for (int j = 0; j < EC; j++) v[qq][j] = __ldcg(p + (int64_t)j * BM);
                }
              }
#pragma unroll
              for (int qq = 0; qq < 2; qq++) {
                const int sgi = g0 + qq;
                if (sgi < nseg) {
#pragma unroll
                  for (int j = 0; j < EC; j++) {
                    const float x = sgi == own ? acc[j] : v[qq][j];
                    sum[j] = sgi == 0 ? x : sum[j] + x;
                  }
                }
              }
            }
#pragma unroll
            for (int j = 0; j < EC; j++) acc[j] = sum[j];
          }
          if (in_rows) wg3::store_c_row<EC>(args.C, args.ldc, row, n0 + c, args.n, args.uplo, alpha, beta, acc);
        }
      }
      wgtc::tc_fence_before();
      wgtc::mbar_arrive_cluster(acc_empty_first + (uint32_t)(b * 8));  // this CTA's rows are drained
    }
  }

  wgtc::tc_fence_before();
  __syncthreads();
  __syncwarp();
  wgtc::cluster_sync();  // no remote arrival or pair MMA is outstanding past this point
  if (warp == 1) {
    __syncwarp();
    wgtc::tc_fence_after();
    wgtc::tmem_dealloc_pair(tmem, 2 * P_BN);
  }
}

// ---- host side ------------------------------------------------------------

// Tensor map of op(A) (rows = m) or of op(B) as its N x K operand (rows = n):
// K-contiguous sources in 64-byte-swizzled boxes of 16 k x box_rows, the others
// in plain boxes of box_rows x 16 k.
bool make_fmap(CUtensorMap *map, const float *ptr, bool kcontig, int64_t rows, int64_t k, int64_t ld, int box_rows) {
  wg_encode_tiled_fn fn = wg_encode_tiled();
  if (!fn) return false;
  cuuint64_t dims[2], strides[1] = {(cuuint64_t)ld * sizeof(float)};
  cuuint32_t box[2], estr[2] = {1, 1};
  if (kcontig) {
    dims[0] = (cuuint64_t)k;
    dims[1] = (cuuint64_t)rows;
    box[0] = 16;
    box[1] = (cuuint32_t)box_rows;
  } else {
    dims[0] = (cuuint64_t)rows;
    dims[1] = (cuuint64_t)k;
    box[0] = (cuuint32_t)box_rows;
    box[1] = 16;
  }
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(ptr), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, kcontig ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

struct FLayout {
  int bn;
  int tiles_m, tiles_n, kt;
  wg3::Plan plan;
};

// Modelled time of a plan, in units of one 16-deep k-block of a 128 x 256 tile:
// whole rounds of kt k-blocks, split rounds of kt/s, the split's overhead, and
// a k-block of a narrower tile costing its share of the MMA time but no less
// than about a third (the operand split and the pipeline's fixed steps).
double plan_time(int G, const wg3::Plan &p, int kt, int bn) {
  const double unit = bn >= 256 ? 1.0 : (bn == 128 ? 0.55 : 0.35);
  double rounds;
  if (p.sk_tiles == 0) {
    rounds = (double)((p.dp_tiles + G - 1) / G) * kt;
  } else {
    const int s = p.sk_split;
    rounds = (double)(p.dp_tiles / G) * kt + (double)(((int64_t)s * p.sk_tiles + G - 1) / G) * ((double)kt / s) +
             wg3::split_overhead(kt, s);
  }
  return rounds * unit;
}

FLayout flayout_of(int G, int64_t m, int64_t n, int64_t k, int bn_force, bool allow_split) {
  FLayout best{0, 0, 0, 0, {0, 0, 0, 1}};
  double best_t = 0.0;
  const int kt = (int)((k + 15) / 16);
  for (int bn : {256, 128, 64}) {
    if (bn_force && bn != bn_force) continue;
    FLayout L;
    L.bn = bn;
    L.tiles_m = (int)((m + BM - 1) / BM);
    L.tiles_n = (int)((n + bn - 1) / bn);
    L.kt = kt;
    L.plan = wg3::plan_tiles(G, L.tiles_m, L.tiles_n, kt, allow_split);
    const double t = plan_time(G, L.plan, kt, bn);
    if (best.bn == 0 || t < best_t * 0.97) {  // prefer the wider tile unless clearly slower
      best = L;
      best_t = t;
    }
  }
  return best;
}

// Scratch of one call: [partials | next_unit | counters | tile_bad | tile_flags];
// everything from next_unit on is zeroed before the launch.
struct FScratch {
  size_t partial_bytes, zero_offset, zero_bytes, total;
};
FScratch fscratch_of(const FLayout &L) {
  FScratch s;
  s.partial_bytes = (size_t)L.plan.sk_tiles * L.plan.sk_split * BM * L.bn * sizeof(float);
  s.zero_offset = s.partial_bytes;
  const size_t tiles = (size_t)L.tiles_m * L.tiles_n;
  s.zero_bytes = (1 + 2 * (size_t)L.plan.sk_tiles + tiles) * sizeof(unsigned);
  s.total = s.zero_offset + s.zero_bytes + 256;
  return s;
}

template <int BN>
cudaError_t launch_bn(cudaStream_t st, int grid, bool a_k, bool b_k, const CUtensorMap &ma, const CUtensorMap &mb,
                      const FArgs &args) {
  using S = FS<BN>;
  auto kern = a_k ? (b_k ? tf32x3_fused<S, 1, 1> : tf32x3_fused<S, 1, 0>)
                  : (b_k ? tf32x3_fused<S, 0, 1> : tf32x3_fused<S, 0, 0>);
  cudaError_t e = wg_kernel_smem(kern, S::SMEM);
  if (e != cudaSuccess) return e;
  kern<<<grid, F_THREADS, S::SMEM, st>>>(ma, mb, args);
  return cudaGetLastError();
}

// The pair kernel's plan: 256 x 256 tiles over sm_count / 2 pairs.
FLayout pair_layout_of(int G, int64_t m, int64_t n, int64_t k, bool allow_split) {
  FLayout L;
  L.bn = P_BN;
  L.tiles_m = (int)((m + 2 * BM - 1) / (2 * BM));
  L.tiles_n = (int)((n + P_BN - 1) / P_BN);
  L.kt = (int)((k + 15) / 16);
  L.plan = wg3::plan_tiles(G / 2 > 0 ? G / 2 : 1, L.tiles_m, L.tiles_n, L.kt, allow_split);
  return L;
}

// Scratch of a pair call: [partials | next_unit | counters | tile_bad | tile_flags],
// counters and tile_bad per 128-row half of each split tile, flags per half tile.
FScratch pair_scratch_of(const FLayout &L) {
  FScratch s;
  s.partial_bytes = (size_t)L.plan.sk_tiles * 2 * L.plan.sk_split * BM * P_BN * sizeof(float);
  s.zero_offset = s.partial_bytes;
  s.zero_bytes = (1 + 4 * (size_t)L.plan.sk_tiles + 2 * (size_t)L.tiles_m * L.tiles_n) * sizeof(unsigned);
  s.total = s.zero_offset + s.zero_bytes + 256;
  return s;
}

}  // namespace

size_t wg_tf32x3_pair_workspace(const wg_device *d, int64_t m, int64_t n, int64_t k) {
  return pair_scratch_of(pair_layout_of(d->sm_count, m, n, k, true)).total;
}

wg_status wg_sgemm_tf32x3_pair(wg_device *d, cudaStream_t st, int transA, int transB, int64_t m, int64_t n, int64_t k,
                               float alpha, const float *A, int64_t lda, const float *B, int64_t ldb, float beta,
                               float *C, int64_t ldc, void *ws, size_t ws_bytes, int uplo) {
  FLayout L = pair_layout_of(d->sm_count, m, n, k, true);
  FScratch sc = pair_scratch_of(L);
  if (sc.total > ws_bytes) {
    L = pair_layout_of(d->sm_count, m, n, k, false);
    sc = pair_scratch_of(L);
    if (sc.total > ws_bytes) return wg_fail(WG_ERR_INVALID_ARGUMENT, "pair 3xTF32 scratch too small");
  }
  const bool a_k = transA != 0, b_k = transB == 0;
  CUtensorMap maps[2];
  if (!make_fmap(&maps[0], A, a_k, m, k, lda, BM) || !make_fmap(&maps[1], B, b_k, n, k, ldb, P_HALF))
    return wg_fail(WG_ERR_CUDA, "cuTensorMapEncodeTiled failed for the pair 3xTF32 operands");
  char *w = static_cast<char *>(ws);
  unsigned *zero = reinterpret_cast<unsigned *>(w + sc.zero_offset);
  WG_CUDA(cudaMemsetAsync(zero, 0, sc.zero_bytes, st));
  const uint32_t epoch = wg_next_epoch(d);
  const wg3::Plan &p = L.plan;
  FArgs args{m, n, k, alpha, beta, C, ldc, d->dwords, L.tiles_m, L.tiles_n, L.kt, p.dp_tiles, p.sk_tiles,
             p.sk_split, p.sk_tiles ? reinterpret_cast<float *>(w) : nullptr, zero, zero + 1,
             zero + 1 + 2 * p.sk_tiles, zero + 1 + 4 * p.sk_tiles, epoch, p.dp_tiles + p.sk_tiles * p.sk_split, uplo};
  {
    wg_launch_scope scope(d, "sgemm_tf32x3_pair", st);
    auto kern = a_k ? (b_k ? tf32x3_fused_pair<1, 1> : tf32x3_fused_pair<1, 0>)
                    : (b_k ? tf32x3_fused_pair<0, 1> : tf32x3_fused_pair<0, 0>);
    WG_CUDA(wg_kernel_smem(kern, P_SMEM));
    kern<<<2 * p.grid, F_THREADS, P_SMEM, st>>>(maps[0], maps[1], args);
    WG_CUDA(cudaGetLastError());
  }
  {
    wg_launch_scope scope(d, "sgemm_simt_fallback", st);
    const wg_gate gate{d->dwords + WG_DW_FALLBACK, d->dwords + WG_DW_FALLBACK, epoch, epoch};
    const wg_tile_mask mask{args.tile_flags, 2 * L.tiles_m, P_BN, epoch};
    WG_CUDA(wg_launch_gemm_simt_masked(st, transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, d->dwords,
                                       &gate, &mask, uplo));
  }
  return WG_OK;
}

bool wg_tf32x3_fused_supported(const wg_device *d, int transA, int transB, int64_t m, int64_t n, int64_t k,
                               const float *A, int64_t lda, const float *B, int64_t ldb) {
  if (d->cc_major != 10 || k < 8 || !wg_encode_tiled()) return false;
  // TMA: 16-byte aligned bases and row strides; coordinates in int range.
  if (reinterpret_cast<uintptr_t>(A) % 16 || reinterpret_cast<uintptr_t>(B) % 16 || lda % 4 || ldb % 4) return false;
  if (m >= ((int64_t)1 << 31) - 512 || n >= ((int64_t)1 << 31) - 512 || k >= ((int64_t)1 << 31) - 64) return false;
  const int64_t tiles = ((m + BM - 1) / BM) * ((n + 63) / 64);
  return tiles < ((int64_t)1 << 30);
}

size_t wg_tf32x3_fused_workspace(const wg_device *d, int64_t m, int64_t n, int64_t k) {
  return fscratch_of(flayout_of(d->sm_count, m, n, k, d->fused_bn, true)).total;
}

wg_status wg_sgemm_tf32x3_fused(wg_device *d, cudaStream_t st, int transA, int transB, int64_t m, int64_t n,
                                int64_t k, float alpha, const float *A, int64_t lda, const float *B, int64_t ldb,
                                float beta, float *C, int64_t ldc, void *ws, size_t ws_bytes, int uplo) {
  FLayout L = flayout_of(d->sm_count, m, n, k, d->fused_bn, true);
  FScratch sc = fscratch_of(L);
  if (sc.total > ws_bytes) {  // no room for the split tiles' partial sums: whole tiles
    L = flayout_of(d->sm_count, m, n, k, d->fused_bn, false);
    sc = fscratch_of(L);
    if (sc.total > ws_bytes) return wg_fail(WG_ERR_INVALID_ARGUMENT, "fused 3xTF32 scratch too small");
  }
  const bool a_k = transA != 0, b_k = transB == 0;
  CUtensorMap maps[2];
  if (!make_fmap(&maps[0], A, a_k, m, k, lda, BM) || !make_fmap(&maps[1], B, b_k, n, k, ldb, L.bn))
    return wg_fail(WG_ERR_CUDA, "cuTensorMapEncodeTiled failed for the fused 3xTF32 operands");
  char *w = static_cast<char *>(ws);
  unsigned *zero = reinterpret_cast<unsigned *>(w + sc.zero_offset);
  WG_CUDA(cudaMemsetAsync(zero, 0, sc.zero_bytes, st));
  const uint32_t epoch = wg_next_epoch(d);
  const wg3::Plan &p = L.plan;
  FArgs args{m, n, k, alpha, beta, C, ldc, d->dwords, L.tiles_m, L.tiles_n, L.kt, p.dp_tiles, p.sk_tiles,
             p.sk_split, p.sk_tiles ? reinterpret_cast<float *>(w) : nullptr, zero, zero + 1,
             zero + 1 + p.sk_tiles, zero + 1 + 2 * p.sk_tiles, epoch, p.dp_tiles + p.sk_tiles * p.sk_split, uplo,
             A, B, lda, ldb};
  {
    // One launch: tiles whose operands the split rules out are computed by the
    // same kernel on the FFMA pipe.
    wg_launch_scope scope(d, "sgemm_tf32x3_fused", st);
    cudaError_t e = L.bn == 256 ? launch_bn<256>(st, p.grid, a_k, b_k, maps[0], maps[1], args)
                  : L.bn == 128 ? launch_bn<128>(st, p.grid, a_k, b_k, maps[0], maps[1], args)
                                : launch_bn<64>(st, p.grid, a_k, b_k, maps[0], maps[1], args);
    WG_CUDA(e);
  }
  return WG_OK;
}
