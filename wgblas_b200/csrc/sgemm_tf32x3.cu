// 3xTF32 sgemm on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// Every fp32 operand x is split into two TF32 values, hi = rna_tf32(x) and
// lo = rna_tf32(x - hi) (x - hi is exact), and the product is taken as
//   A*B ~= A_hi*B_hi + A_hi*B_lo + A_lo*B_hi
// with fp32 accumulation in TMEM: the representation error is ~3*2^-22 of each
// |a||b| and the dropped lo*lo term ~2^-22, inside the north-star bound
// 2*K*2^-24*(|A||B| + |C|) for K >= 6 (the dispatcher uses it for K >= 64).
// The alpha/beta epilogue is the reference's (src/shaders/sgemm_large.wgsl:299-304)
// in fp32 with the beta term fused.
//
// Two launches per call (plus the gated fallback):
//  1. tf32x3_pack: reads op(A) and op(B) in any transpose / leading dimension,
//     writes K-major, zero-padded hi and lo operands to the scratch workspace,
//     and flags (writes the call's epoch into a device word) any element that
//     is not finite or whose magnitude lies outside [2^-50, 2^50] — there the
//     split loses its accuracy (subnormal lo parts) or IEEE semantics (Inf*0 in
//     a cross term).
//  2. tf32x3_mma: a persistent grid, one CTA per SM, over 128 x BN tiles of C.
//     Warp 0 streams the four operand tiles of each k-block into a
//     STAGES-deep shared-memory ring with TMA (no multicast); warp 1 issues
//     three tcgen05.mma.kind::tf32 per 8-wide k step into one of two TMEM
//     accumulators; warps 2-5 read the other accumulator with tcgen05.ld and
//     store C column by column (32 rows = 128 contiguous bytes per warp store),
//     so a tile's epilogue overlaps the next tile's main loop. Tiles are
//     visited in groups of GROUP_M tile rows for L2 reuse.
//     Work split: units are handed out in raster order from a work counter
//     (each CTA's first is its blockIdx.x), so CTAs running together work on
//     neighbouring tiles for L2 reuse and an SM slowed by other kernels
//     (operand splits of the next panel, a broadcast) simply takes fewer; the
//     leftover tiles of a partial last wave are cut into s equal k-segments
//     when that shortens the wave (plan_of), numbered so units handed out
//     together share a k range. A split tile is finished by whichever segment
//     arrives last (a per-tile atomic counter): the others leave their fp32
//     partial sums in the workspace, and the last adds all segments in k order
//     — no CTA ever waits for another, and the result does not depend on
//     arrival order. Without room for the partial sums all tiles go whole.
//     gemmtr calls skip the units whose tile has no element in the triangle
//     and mask the diagonal tiles' stores.
//  When the pack flagged the operands (the gate: a flag word holding the
//  call's epoch) the MMA kernel computes C itself on the FFMA pipe instead,
//  with all eight warps running the SIMT GEMM's tile (simt_tile.cuh), so the
//  result has the reference's IEEE semantics and the FFMA kernel's bits. An
//  unflagged call launches nothing else.
#include <cuda.h>

#include <mutex>

#include "internal.h"
#include "simt_tile.cuh"
#include "tcgen05.cuh"
#include "tf32x3_common.cuh"

namespace {

using wg3::BM;
using wg3::EPI_WARPS;
using wg3::WAIT_BUDGET;
using wg3::GROUP_M;
using wg3::MAX_SEG;
using wg3::UQ;
using wg3::Unit;
using wg3::rna_tf32;
using wg3::split_ok;
using wg3::epi_bar;
using wg3::epi_all;
using wg3::mbar_arrive;
using wg3::Plan;
using wg3::split_overhead;
// Producer, MMA issuer, EPI_WARPS epilogue warps and two more that only the
// FFMA fallback uses (its tile needs 256 threads; one CTA per SM either way, at
// 255 registers a thread).
constexpr int THREADS = 32 * (2 + EPI_WARPS + 2);
static_assert(THREADS == wgsimt::NT, "the fallback runs the SIMT tile with every thread");
constexpr int SEG_GROUP = 2;  // partial-sum segments the fixup loads at once

// Kernel shape: BN columns of C per CTA, BK floats of K per pipeline stage
// (BK * 4 bytes = the swizzle span: 128 -> SWIZZLE_128B, 64 -> SWIZZLE_64B).
template <int BN_, int BK_, int STAGES_>
struct Shape {
  static constexpr int BN = BN_, BK = BK_, STAGES = STAGES_;
  static constexpr int ROW_BYTES = BK * 4;
  static constexpr int A_TILE = BM * BK * 4;  // bytes of one A operand tile
  static constexpr int B_TILE = BN * BK * 4;
  static constexpr int STAGE = 2 * A_TILE + 2 * B_TILE;  // A_hi, A_lo, B_hi, B_lo
  static constexpr int TMEM_COLS = BN;  // fp32 accumulator: 128 lanes x BN columns
  static constexpr size_t SMEM = 1024 /*alignment slack*/ + (size_t)STAGES * STAGE + 256 /*barriers*/;
  static_assert(A_TILE % 1024 == 0 && B_TILE % 1024 == 0, "tiles must keep 1024-byte alignment");
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "UMMA N for M=128 is a multiple of 16 up to 256");
  static_assert(ROW_BYTES == 64 || ROW_BYTES == 128, "swizzle span");
};

using Sh = Shape<256, 16, 4>;  // 48 KB stages, four deep

struct PackArgs {
  const float *src;
  int64_t ld;
  int kcontig;    // 1: element (r, p) at src[r*ld + p]; 0: at src[r + p*ld]
  int64_t rows;   // real rows (m for A, n for B)
  int64_t rows_p; // padded rows
  float *hi, *lo; // rows_p x kp, row-major (K contiguous)
  int64_t tiles_r;
  unsigned *flag; // set to `epoch` when an element rules the split out
  uint32_t epoch;
};

// One 32 x 32 (rows x k) tile per 256-thread block; blocks [0, tilesA) pack A,
// the rest pack B. Writes are 128-byte rows of K; reads are coalesced along
// whichever dimension the source stores contiguously (through shared memory
// when that is the row dimension).
__global__ void __launch_bounds__(256) tf32x3_pack(PackArgs a, PackArgs b, int64_t k, int64_t kp,
                                                   int64_t tiles_a, unsigned *counters, int64_t n_counters,
                                                   unsigned *next_unit) {
  __shared__ float tile[32][33];
  wg_pdl_trigger();  // the MMA kernel may set itself up while the last blocks split
  // The split-tile counters and the work counter of the MMA launch that follows start at zero.
  if (blockIdx.x == 0) {
    for (int64_t i = threadIdx.x; i < n_counters; i += blockDim.x) counters[i] = 0;
    if (next_unit && threadIdx.x == 0) *next_unit = 0;
  }
  const bool is_a = blockIdx.x < tiles_a;
  const PackArgs &P = is_a ? a : b;
  const int64_t t = is_a ? blockIdx.x : blockIdx.x - tiles_a;
  const int64_t tiles_k = kp / 32;
  const int64_t r0 = (t / tiles_k) * 32, p0 = (t % tiles_k) * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // ty in [0, 8)
  bool bad = false;
  float v[4];
  if (P.kcontig) {
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int64_t r = r0 + ty + 8 * i, p = p0 + tx;
      v[i] = (r < P.rows && p < k) ? P.src[r * P.ld + p] : 0.0f;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const int64_t p = p0 + ty + 8 * i, r = r0 + tx;
      tile[ty + 8 * i][tx] = (r < P.rows && p < k) ? P.src[r + p * P.ld] : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 4; i++) v[i] = tile[tx][ty + 8 * i];
  }
#pragma unroll
  for (int i = 0; i < 4; i++) {
    const int64_t r = r0 + ty + 8 * i, p = p0 + tx;
    const float x = v[i];
    bad |= !split_ok(x);
    const float h = rna_tf32(x);
    const float l = rna_tf32(x - h);
    P.hi[r * kp + p] = h;
    P.lo[r * kp + p] = l;
  }
  if (__any_sync(0xffffffffu, bad) && tx == 0) *(volatile unsigned *)P.flag = P.epoch;
}


struct MmaArgs {
  int64_t m, n, k;
  float alpha, beta;
  float *C;
  int64_t ldc;
  unsigned *dwords;          // WG_DW_ERROR receives the wait-timeout bits
  wg_gate gate;              // open: the operands ruled the split out, the FFMA kernel computes C
  int tiles_m, tiles_n, kt;  // tile grid and k-blocks per tile
  int dp_tiles;              // tiles [0, dp_tiles) are taken whole, round-robin over the grid
  int sk_tiles;              // the remaining tiles, each split into sk_split k-segments
  int sk_split;
  float *partials;           // split tiles: [sk_tiles * sk_split][BN][BM] partial sums
  unsigned *counters;        // split tiles: one arrival counter each
  unsigned *next_unit;       // work counter: units handed out beyond the first gridDim.x
  int units;                 // dp_tiles + sk_tiles * sk_split
  int uplo;                  // WG_UPLO_*: tiles with no element in the triangle are skipped
  // The caller's operands, for the FFMA fallback.
  const float *A, *B;
  int64_t lda, ldb;
  int transA, transB;
};

// C for a call whose operands the split ruled out, on the FFMA pipe: the SIMT
// GEMM's 128 x 128 tiles, grid-stride, every thread of the block, shared memory
// from the (unused) operand ring.
__device__ __forceinline__ void ffma_fallback(const MmaArgs &a, uint8_t *smem) {
  using namespace wgsimt;
  float *As = reinterpret_cast<float *>(smem);
  float *Bs = As + 2 * wgsimt::BK * lda_s<float>();
  const int64_t kk = a.alpha == 0.0f ? 0 : a.k;
  const int64_t tiles_m = (a.m + wgsimt::BM - 1) / wgsimt::BM, tiles = tiles_m * ((a.n + wgsimt::BN - 1) / wgsimt::BN);
  const wg_tile_mask all{nullptr, 1, 1, 0u};
  for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x) {
    const int64_t m0 = (t % tiles_m) * wgsimt::BM, n0 = (t / tiles_m) * wgsimt::BN;
    if (wg_tile_outside(a.uplo, m0, wgsimt::BM, n0, wgsimt::BN)) continue;
    if (a.transA) {
      if (a.transB)
        tile<float, 1, 1>(m0, n0, a.m, a.n, kk, a.alpha, a.A, a.lda, a.B, a.ldb, a.beta, a.C, a.ldc, all, a.uplo, As, Bs);
      else
        tile<float, 1, 0>(m0, n0, a.m, a.n, kk, a.alpha, a.A, a.lda, a.B, a.ldb, a.beta, a.C, a.ldc, all, a.uplo, As, Bs);
    } else {
      if (a.transB)
        tile<float, 0, 1>(m0, n0, a.m, a.n, kk, a.alpha, a.A, a.lda, a.B, a.ldb, a.beta, a.C, a.ldc, all, a.uplo, As, Bs);
      else
        tile<float, 0, 0>(m0, n0, a.m, a.n, kk, a.alpha, a.A, a.lda, a.B, a.ldb, a.beta, a.C, a.ldc, all, a.uplo, As, Bs);
    }
  }
}

template <class S>
__global__ void __launch_bounds__(THREADS, 1)
tf32x3_mma(const __grid_constant__ CUtensorMap map_ahi, const __grid_constant__ CUtensorMap map_alo,
           const __grid_constant__ CUtensorMap map_bhi, const __grid_constant__ CUtensorMap map_blo,
           const MmaArgs args) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t base = wgtc::smem_addr(smem_raw);
  uint8_t *smem = smem_raw + ((1024 - (base & 1023)) & 1023);  // 1024-byte aligned ring
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + (size_t)S::STAGES * S::STAGE);
  uint64_t *empty = full + S::STAGES;
  uint64_t *acc_full = empty + S::STAGES;  // [2]: accumulator b holds a finished unit
  uint64_t *acc_empty = acc_full + 2;      // [2]: the epilogue has drained accumulator b
  uint64_t *uq_full = acc_empty + 2;       // [UQ]: the producer has written unit slot i
  uint64_t *uq_empty = uq_full + UQ;       // [UQ]: the MMA issuer and the epilogue have read it
  volatile int *uq = reinterpret_cast<volatile int *>(uq_empty + UQ);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(const_cast<int *>(uq) + UQ);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);
  volatile unsigned *last_flag = reinterpret_cast<volatile unsigned *>(tmem_slot + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S::STAGES; s++) {
      wgtc::mbar_init(&full[s], 1);
      wgtc::mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; b++) {
      wgtc::mbar_init(&acc_full[b], 1);
      wgtc::mbar_init(&acc_empty[b], 32 * EPI_WARPS);
    }
    for (int i = 0; i < UQ; i++) {
      wgtc::mbar_init(&uq_full[i], 1);
      wgtc::mbar_init(&uq_empty[i], 2);
    }
    *abort_flag = 0;
    wgtc::fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    wgtc::prefetch_tensormap(&map_ahi);
    wgtc::prefetch_tensormap(&map_alo);
    wgtc::prefetch_tensormap(&map_bhi);
    wgtc::prefetch_tensormap(&map_blo);
  }
  if (warp == 1) {
    wgtc::tmem_alloc(tmem_slot, 2 * S::TMEM_COLS);  // two accumulators
    wgtc::tmem_relinquish();
  }
  wgtc::tc_fence_before();
  __syncthreads();
  wgtc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // The setup above overlaps the split pass's last blocks (programmatic
  // launch); everything below reads what it wrote: operands, counters, gate.
  wg_pdl_wait();
  if (wg_gate_open(args.gate)) {
    // Operands ruled out by the split (the gate, the same for every thread): C
    // comes from the FFMA pipe instead, with the reference's IEEE semantics.
    if (blockIdx.x == 0 && threadIdx.x == 0) atomicAdd(args.dwords + WG_DW_FALLBACKS, 1u);
    ffma_fallback(args, smem);
  } else if (warp == 0 && lane == 0) {
    // ---- TMA producer: takes units (its first is blockIdx.x, later ones from the
    // work counter, so SMs slowed by other kernels take fewer), hands each to the
    // other roles, and streams its k-blocks into one continuous ring ----
    int64_t g = 0;
    bool ok = true;
    for (int n = 0; ok; n++) {
      const int slot = n % UQ;
      const uint32_t uph = (uint32_t)(n / UQ) & 1u;
      int un = n == 0 ? (int)blockIdx.x : (int)gridDim.x + (int)atomicAdd(args.next_unit, 1u);
      // gemmtr: tiles with no element in the triangle are not computed at all.
      while (args.uplo != WG_UPLO_FULL && un < args.units) {
        int tm0, tn0;
        wg3::raster(args, wg3::decode(args, un).t, tm0, tn0);
        if (!wg_tile_outside(args.uplo, (int64_t)tm0 * BM, BM, (int64_t)tn0 * S::BN, S::BN)) break;
        un = (int)gridDim.x + (int)atomicAdd(args.next_unit, 1u);
      }
      if (un >= args.units) un = -1;  // no work left: tells the other roles to stop
      if (!wgtc::mbar_wait_bounded(&uq_empty[slot], uph ^ 1u, WAIT_BUDGET) || *abort_flag) {
        atomicOr(args.dwords + WG_DW_ERROR, WG_DERR_TMA_WAIT);
        *abort_flag = 1;
        break;
      }
      uq[slot] = un;
      mbar_arrive(&uq_full[slot]);
      if (un < 0) break;
      const Unit u = wg3::decode(args, un);
      int tm, tn;
      wg3::raster(args, u.t, tm, tn);
      for (int kb = u.kb0; kb < u.kb1; kb++, g++) {
        const int s = (int)(g % S::STAGES);
        const uint32_t ph = (uint32_t)(g / S::STAGES) & 1u;
        if (!wgtc::mbar_wait_bounded(&empty[s], ph ^ 1u, WAIT_BUDGET) || *abort_flag) {
          atomicOr(args.dwords + WG_DW_ERROR, WG_DERR_TMA_WAIT);
          *abort_flag = 1;
          ok = false;
          break;
        }
        uint8_t *st = smem + (size_t)s * S::STAGE;
        wgtc::mbar_arrive_expect_tx(&full[s], S::STAGE);
        const int kc = kb * S::BK;
        wgtc::tma_load_2d(st, &map_ahi, &full[s], kc, tm * BM);
        wgtc::tma_load_2d(st + S::A_TILE, &map_alo, &full[s], kc, tm * BM);
        wgtc::tma_load_2d(st + 2 * S::A_TILE, &map_bhi, &full[s], kc, tn * S::BN);
        wgtc::tma_load_2d(st + 2 * S::A_TILE + S::B_TILE, &map_blo, &full[s], kc, tn * S::BN);
      }
    }
    // Let every copy this thread issued land before the CTA can exit.
    for (int64_t q = g - S::STAGES > 0 ? g - S::STAGES : 0; q < g; q++)
      wgtc::mbar_wait_bounded(&full[q % S::STAGES], (uint32_t)(q / S::STAGES) & 1u, WAIT_BUDGET);
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer ----
    constexpr uint32_t idesc = wgtc::idesc_tf32(BM, S::BN);
    int64_t g = 0;
    bool ok = true;
    for (int n_units = 0; ok; n_units++) {
      const int slot = n_units % UQ;
      if (!wgtc::mbar_wait_bounded(&uq_full[slot], (uint32_t)(n_units / UQ) & 1u, WAIT_BUDGET) || *abort_flag) {
        atomicOr(args.dwords + WG_DW_ERROR, WG_DERR_MMA_WAIT);
        *abort_flag = 1;
        break;
      }
      const int un = uq[slot];
      mbar_arrive(&uq_empty[slot]);
      if (un < 0) break;
      const Unit u = wg3::decode(args, un);
      const int b = n_units & 1;
      const uint32_t use = (uint32_t)(n_units >> 1);
      if (!wgtc::mbar_wait_bounded(&acc_empty[b], (use & 1u) ^ 1u, WAIT_BUDGET) || *abort_flag) {
        atomicOr(args.dwords + WG_DW_ERROR, WG_DERR_MMA_WAIT);
        *abort_flag = 1;
        break;
      }
      wgtc::tc_fence_after();
      const uint32_t d_tmem = tmem + (uint32_t)(b * S::TMEM_COLS);
      for (int kb = u.kb0; kb < u.kb1; kb++, g++) {
        const int s = (int)(g % S::STAGES);
        const uint32_t ph = (uint32_t)(g / S::STAGES) & 1u;
        if (!wgtc::mbar_wait_bounded(&full[s], ph, WAIT_BUDGET) || *abort_flag) {
          atomicOr(args.dwords + WG_DW_ERROR, WG_DERR_TMA_WAIT);
          *abort_flag = 1;
          ok = false;
          break;
        }
        wgtc::tc_fence_after();
        const uint32_t st = wgtc::smem_addr(smem + (size_t)s * S::STAGE);
        const uint32_t a_hi = st, a_lo = st + S::A_TILE, b_hi = st + 2 * S::A_TILE,
                       b_lo = st + 2 * S::A_TILE + S::B_TILE;
#pragma unroll
        for (int kk = 0; kk < S::BK / 8; kk++) {
          const uint32_t off = kk * 32;  // 8 tf32 = 32 bytes along K inside the swizzle span
          const uint64_t dah = wgtc::smem_desc_kmajor(a_hi + off, S::ROW_BYTES);
          const uint64_t dal = wgtc::smem_desc_kmajor(a_lo + off, S::ROW_BYTES);
          const uint64_t dbh = wgtc::smem_desc_kmajor(b_hi + off, S::ROW_BYTES);
          const uint64_t dbl = wgtc::smem_desc_kmajor(b_lo + off, S::ROW_BYTES);
          const uint32_t acc0 = (kb > u.kb0 || kk > 0) ? 1u : 0u;
          wgtc::mma_tf32(d_tmem, dal, dbh, idesc, acc0);  // small terms first
          wgtc::mma_tf32(d_tmem, dah, dbl, idesc, 1u);
          wgtc::mma_tf32(d_tmem, dah, dbh, idesc, 1u);
        }
        wgtc::mma_commit(&empty[s]);  // frees the stage once these MMAs have read it
      }
      wgtc::mma_commit(&acc_full[b]);  // accumulator b complete once all its MMAs finish
    }
  } else if (warp >= 2 && warp < 2 + EPI_WARPS) {
    // ---- epilogue: TMEM -> registers -> C (or a partial-sum slot) ----
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int row_in_tile = q * 32 + lane;
    const float alpha = args.alpha, beta = args.beta;
    for (int n_units = 0;; n_units++) {
      const int slot = n_units % UQ;
      const bool got = wgtc::mbar_wait_bounded(&uq_full[slot], (uint32_t)(n_units / UQ) & 1u, WAIT_BUDGET);
      const int un = got ? uq[slot] : -1;
      // One decision for all 128 epilogue threads (tcgen05.ld is warp-collective and
      // the partial-sum path below meets at a named barrier); it also means every
      // thread has read the slot before it is released.
      if (!epi_all(got && *abort_flag == 0)) {
        if (!got) atomicOr(args.dwords + WG_DW_ERROR, WG_DERR_MMA_WAIT);
        *abort_flag = 1;
        break;
      }
      if (threadIdx.x == 64) mbar_arrive(&uq_empty[slot]);
      if (un < 0) break;
      const Unit u = wg3::decode(args, un);
      const int b = n_units & 1;
      const uint32_t use = (uint32_t)(n_units >> 1);
      const bool ready = wgtc::mbar_wait_bounded(&acc_full[b], use & 1u, WAIT_BUDGET);
      if (!epi_all(ready && *abort_flag == 0)) {
        if (!ready) atomicOr(args.dwords + WG_DW_ERROR, WG_DERR_MMA_WAIT);
        *abort_flag = 1;
        break;
      }
      wgtc::tc_fence_after();
      int tm, tn;
      wg3::raster(args, u.t, tm, tn);
      const int64_t row = (int64_t)tm * BM + row_in_tile;
      const int64_t n0 = (int64_t)tn * S::BN;
      const uint32_t trow = tmem + (uint32_t)(b * S::TMEM_COLS) + ((uint32_t)(q * 32) << 16);
      const bool whole = u.seg < 0;
      bool finish = whole;
      const int local = u.t - args.dp_tiles;
      if (!whole) {
        // Leave this segment's partial sums, then count arrivals on the tile.
        float *part = args.partials + ((int64_t)local * args.sk_split + u.seg) * S::BN * BM + row_in_tile;
        for (int c = 0; c < S::BN; c += 32) {
          uint32_t r[32];
          wgtc::tmem_ld_32x32b_x32(trow + (uint32_t)c, r);
          wgtc::tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; j++) part[(int64_t)(c + j) * BM] = __uint_as_float(r[j]);
        }
        __threadfence();
        epi_bar();
        if (threadIdx.x == 64) {
          const unsigned prev = atomicAdd(args.counters + local, 1u);
          const bool last = prev == (unsigned)(args.sk_split - 1);
          if (last) args.counters[local] = 0;  // ready for the next call on this workspace
          *last_flag = last ? 1u : 0u;
          __threadfence();
        }
        epi_bar();
        finish = *last_flag != 0;
        if (finish) __threadfence();  // order the reads of the other segments' partial sums
      }
      if (finish) {
        // Segments of this tile in k order; this CTA's own comes from TMEM. The
        // partial sums of SEG_GROUP segments (32 columns each) are loaded together,
        // and the 32 old C values of a chunk are loaded before any is written, so a
        // chunk costs one memory round trip per SEG_GROUP segments (plus one for C)
        // instead of one per value.
        const int nseg = whole ? 1 : args.sk_split;
        const int own = whole ? 0 : u.seg;
        const float *part0 = whole ? nullptr
                                   : args.partials + (int64_t)local * args.sk_split * S::BN * BM + row_in_tile;
        const bool in_rows = row < args.m;
        for (int c = 0; c < S::BN; c += 32) {
          uint32_t r[32];
          wgtc::tmem_ld_32x32b_x32(trow + (uint32_t)c, r);
          wgtc::tmem_ld_wait();
          float acc[32];
#pragma unroll
          for (int j = 0; j < 32; j++) acc[j] = __uint_as_float(r[j]);
          if (nseg > 1) {
            float sum[32];
            for (int g0 = 0; g0 < nseg; g0 += SEG_GROUP) {
              float v[SEG_GROUP][32];
#pragma unroll
              for (int q = 0; q < SEG_GROUP; q++) {
                const int sgi = g0 + q;
                if (sgi < nseg && sgi != own) {
                  const float *p = part0 + ((int64_t)sgi * S::BN + c) * BM;
#pragma unroll
                  for (int j = 0; j < 32; j++) v[q][j] = __ldcg(p + (int64_t)j * BM);
                }
              }
#pragma unroll
              for (int q = 0; q < SEG_GROUP; q++) {
                const int sgi = g0 + q;
                if (sgi < nseg) {
#pragma unroll
                  for (int j = 0; j < 32; j++) {
                    const float x = sgi == own ? acc[j] : v[q][j];
                    sum[j] = sgi == 0 ? x : sum[j] + x;
                  }
                }
              }
            }
#pragma unroll
            for (int j = 0; j < 32; j++) acc[j] = sum[j];
          }
          if (in_rows) wg3::store_c_row<32>(args.C, args.ldc, row, n0 + c, args.n, args.uplo, alpha, beta, acc);
        }
      }
      wgtc::tc_fence_before();
      mbar_arrive(&acc_empty[b]);  // accumulator b may be refilled
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

// ---- host side ------------------------------------------------------------
// ---- host side ------------------------------------------------------------

wg_encode_tiled_fn encode_fn() { return wg_encode_tiled(); }

// Tensor map of a rows x kp row-major fp32 operand, boxes of box_rows x BK.
bool make_map(CUtensorMap *map, float *ptr, int64_t rows, int64_t kp, int box_rows) {
  wg_encode_tiled_fn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)kp, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)kp * sizeof(float)};
  cuuint32_t box[2] = {(cuuint32_t)Sh::BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  const CUtensorMapSwizzle sw = Sh::ROW_BYTES == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, ptr, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
            sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

struct Layout {
  int64_t mp, np, kp;
  size_t a_bytes, b_bytes, operands;  // split operands
  int tiles_m, tiles_n, kt;
};

Layout layout_of(int64_t m, int64_t n, int64_t k) {
  Layout L;
  L.mp = (m + BM - 1) / BM * BM;
  L.np = (n + Sh::BN - 1) / Sh::BN * Sh::BN;
  L.kp = (k + 31) / 32 * 32;  // the pack kernel's tile; a multiple of BK
  L.a_bytes = (size_t)L.mp * L.kp * sizeof(float);
  L.b_bytes = (size_t)L.np * L.kp * sizeof(float);
  L.operands = 2 * L.a_bytes + 2 * L.b_bytes;
  L.tiles_m = (int)(L.mp / BM);
  L.tiles_n = (int)(L.np / Sh::BN);
  L.kt = (int)(L.kp / Sh::BK);
  return L;
}

Plan plan_of(int G, const Layout &L, bool allow_split) {
  return wg3::plan_tiles(G, L.tiles_m, L.tiles_n, L.kt, allow_split);
}

// Scratch after the split operands: the partial sums of the split tiles, then
// one arrival counter per split tile (plus slack for alignment).
size_t sk_partial_bytes(const Plan &p) { return (size_t)p.sk_tiles * p.sk_split * BM * Sh::BN * sizeof(float); }
size_t sk_bytes(const Plan &p) { return sk_partial_bytes(p) + (size_t)p.sk_tiles * sizeof(unsigned) + 256; }

// Splits op(A) (tiles_a blocks) and/or op(B) on stream `s`, zeroing n_counters
// split-tile counters and the MMA launch's work counter (when given) first.
wg_status launch_pack(wg_device *d, cudaStream_t s, const PackArgs &pa, const PackArgs &pb, int64_t k, int64_t kp,
                      unsigned *counters, int64_t n_counters, unsigned *next_unit) {
  const int64_t blocks = pa.tiles_r + pb.tiles_r;
  if (blocks == 0) return WG_OK;
  wg_launch_scope scope(d, "sgemm_tf32x3_pack", s);
  tf32x3_pack<<<(unsigned)blocks, 256, 0, s>>>(pa, pb, k, kp, pa.tiles_r, counters, n_counters, next_unit);
  WG_CUDA(cudaGetLastError());
  return WG_OK;
}

// The MMA launch over split operands already in place, on d->stream; when
// `gate` is open it computes C on the FFMA pipe instead. With `pdl` the split
// pass is the launch right before it on the stream, and the kernel sets itself
// up while that pass finishes (programmatic dependent launch). The last
// wave's tiles are split along k when sk_room bytes at `sk` hold the plan's
// partial sums and counters (counters at sk + partial_room, zeroed
// beforehand), whole otherwise. next_unit is the work counter, zeroed beforehand.
wg_status launch_mma(wg_device *d, int transA, int transB, int64_t m, int64_t n, int64_t k, float alpha,
                     const float *A, int64_t lda, const float *B, int64_t ldb, float beta, float *C, int64_t ldc,
                     float *ahi, float *alo, float *bhi, float *blo, char *sk, size_t partial_room,
                     int64_t counter_room, unsigned *next_unit, const wg_gate &gate, int uplo, bool pdl) {
  const Layout L = layout_of(m, n, k);
  const int G = d->sm_count;
  Plan plan = plan_of(G, L, true);
  if (sk_partial_bytes(plan) > partial_room || plan.sk_tiles > counter_room) plan = plan_of(G, L, false);
  const bool split = plan.sk_tiles > 0;
  float *partials = split ? reinterpret_cast<float *>(sk) : nullptr;
  unsigned *counters = split ? reinterpret_cast<unsigned *>(sk + partial_room) : nullptr;
  CUtensorMap maps[4];
  if (!make_map(&maps[0], ahi, L.mp, L.kp, BM) || !make_map(&maps[1], alo, L.mp, L.kp, BM) ||
      !make_map(&maps[2], bhi, L.np, L.kp, Sh::BN) || !make_map(&maps[3], blo, L.np, L.kp, Sh::BN))
    return wg_fail(WG_ERR_CUDA, "cuTensorMapEncodeTiled failed for the 3xTF32 operands");
  MmaArgs args{m, n, k, alpha, beta, C, ldc, d->dwords, gate, L.tiles_m, L.tiles_n, L.kt, plan.dp_tiles,
               plan.sk_tiles, plan.sk_split, partials, counters, next_unit,
               plan.dp_tiles + plan.sk_tiles * plan.sk_split, uplo, A, B, lda, ldb, transA, transB};
  auto kern = tf32x3_mma<Sh>;
  WG_CUDA(wg_kernel_smem(kern, Sh::SMEM));
  {
    wg_launch_scope scope(d, "sgemm_tf32x3_mma");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)plan.grid);
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = Sh::SMEM;
    cfg.stream = d->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    WG_CUDA(cudaLaunchKernelEx(&cfg, kern, maps[0], maps[1], maps[2], maps[3], args));
  }
  return WG_OK;
}

// op(A)(i, p): K-contiguous when transA (A[p + i*lda]); op(B)(p, j) as row j of
// the N x K operand: K-contiguous when !transB (B[p + j*ldb]).
PackArgs pack_a_args(int transA, const float *A, int64_t lda, int64_t m, const Layout &L, float *hi, float *lo,
                     unsigned *flag, uint32_t epoch) {
  return PackArgs{A, lda, transA ? 1 : 0, m, L.mp, hi, lo, (L.mp / 32) * (L.kp / 32), flag, epoch};
}
PackArgs pack_b_args(int transB, const float *B, int64_t ldb, int64_t n, const Layout &L, float *hi, float *lo,
                     unsigned *flag, uint32_t epoch) {
  return PackArgs{B, ldb, transB ? 0 : 1, n, L.np, hi, lo, (L.np / 32) * (L.kp / 32), flag, epoch};
}
PackArgs no_pack() { return PackArgs{nullptr, 0, 0, 0, 0, nullptr, nullptr, 0, nullptr, 0}; }

// Scratch of a panelled product: op(A)'s split, two alternating op(B) split
// buffers sized for the widest panel, and the split-K room of the most
// demanding panel.
struct ProductLayout {
  size_t a_region, slot_bytes, partial_room;
  int64_t counter_room;
  size_t total;
};

ProductLayout product_layout(int G, int64_t m, int64_t k, const int64_t *widths, size_t count) {
  ProductLayout P{0, 0, 0, 0, 0};
  int64_t widest = 0;
  for (size_t i = 0; i < count; i++) widest = widths[i] > widest ? widths[i] : widest;
  const Layout W = layout_of(m, widest > 0 ? widest : 1, k);
  P.a_region = 2 * W.a_bytes;
  P.slot_bytes = 2 * W.b_bytes;
  for (size_t i = 0; i < count; i++) {
    const Plan p = plan_of(G, layout_of(m, widths[i], k), true);
    P.partial_room = sk_partial_bytes(p) > P.partial_room ? sk_partial_bytes(p) : P.partial_room;
    P.counter_room = p.sk_tiles > P.counter_room ? p.sk_tiles : P.counter_room;
  }
  P.total = P.a_region + 2 * P.slot_bytes + P.partial_room + (size_t)P.counter_room * sizeof(unsigned) + 256;
  return P;
}

}  // namespace

size_t wg_tf32x3_workspace_bytes(int64_t m, int64_t n, int64_t k) { return layout_of(m, n, k).operands; }

size_t wg_tf32x3_workspace_bytes_sk(const wg_device *d, int64_t m, int64_t n, int64_t k) {
  const Layout L = layout_of(m, n, k);
  return L.operands + sk_bytes(plan_of(d->sm_count, L, true));
}

double wg_tf32x3_cost(int G, int64_t m, int64_t n, int64_t k) {
  const Layout L = layout_of(m, n, k);
  const Plan p = plan_of(G, L, true);
  if (p.sk_tiles == 0) return (double)((p.dp_tiles + G - 1) / G) * L.kt;  // whole tiles only
  const int s = p.sk_split;
  const int64_t rounds = ((int64_t)s * p.sk_tiles + G - 1) / G;
  return (double)(p.dp_tiles / G) * L.kt + (double)rounds * ((double)L.kt / s) + split_overhead(L.kt, s);
}

bool wg_tf32x3_supported(const wg_device *d, int64_t m, int64_t n, int64_t k) {
  if (d->cc_major != 10 || k < 8 || !encode_fn()) return false;
  const Layout L = layout_of(m, n, k);
  // TMA coordinates are 32-bit; tile and iteration counts stay in int range.
  return L.mp < ((int64_t)1 << 31) && L.np < ((int64_t)1 << 31) && L.kp < ((int64_t)1 << 31) &&
         (int64_t)L.tiles_m * L.tiles_n < ((int64_t)1 << 30);
}

extern "C" wg_status wg_sgemm_tc_plan(int sm_count, int64_t m, int64_t n, int64_t k, wg_tc_plan *out) {
  if (!out) return wg_fail(WG_ERR_INVALID_ARGUMENT, "out is NULL");
  if (sm_count <= 0 || m <= 0 || n <= 0 || k < 8)
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "sm_count, m and n must be positive and k >= 8");
  const Layout L = layout_of(m, n, k);
  if ((int64_t)L.tiles_m * L.tiles_n >= ((int64_t)1 << 30))
    return wg_fail(WG_ERR_NOT_SUPPORTED, "too many tiles");
  const Plan p = plan_of(sm_count, L, true);
  out->tiles_m = L.tiles_m;
  out->tiles_n = L.tiles_n;
  out->k_blocks = L.kt;
  out->grid = p.grid;
  out->whole_tiles = p.dp_tiles;
  out->split_tiles = p.sk_tiles;
  out->split_segments = p.sk_split;
  out->workspace_bytes = L.operands + sk_bytes(p);
  return WG_OK;
}

uint32_t wg_next_epoch(wg_device *d) {
  if (++d->epoch == 0) d->epoch = 1;
  return d->epoch;
}

wg_encode_tiled_fn wg_encode_tiled() {
  static wg_encode_tiled_fn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<wg_encode_tiled_fn>(p);
  });
  return fn;
}

wg_status wg_sgemm_tf32x3(wg_device *d, int transA, int transB, int64_t m, int64_t n, int64_t k, float alpha,
                          const float *A, int64_t lda, const float *B, int64_t ldb, float beta, float *C,
                          int64_t ldc, void *ws, size_t ws_bytes, int uplo) {
  const Layout L = layout_of(m, n, k);
  float *ahi = static_cast<float *>(ws);
  float *alo = ahi + L.a_bytes / sizeof(float);
  float *bhi = alo + L.a_bytes / sizeof(float);
  float *blo = bhi + L.b_bytes / sizeof(float);
  // Split the last wave's tiles when the workspace has room for their partial sums.
  Plan plan = plan_of(d->sm_count, L, true);
  if (ws_bytes < L.operands + sk_bytes(plan)) plan = plan_of(d->sm_count, L, false);
  char *sk = static_cast<char *>(ws) + L.operands;
  const size_t partial_room = sk_partial_bytes(plan);
  unsigned *counters = reinterpret_cast<unsigned *>(sk + partial_room);
  const uint32_t epoch = wg_next_epoch(d);
  unsigned *flag = d->dwords + WG_DW_FALLBACK;
  unsigned *next_unit = d->dwords + WG_DW_NEXT_UNIT0;
  wg_status st = launch_pack(d, d->stream, pack_a_args(transA, A, lda, m, L, ahi, alo, flag, epoch),
                             pack_b_args(transB, B, ldb, n, L, bhi, blo, flag, epoch), k, L.kp, counters,
                             plan.sk_tiles, next_unit);
  if (st != WG_OK) return st;
  const wg_gate gate{flag, flag, epoch, epoch};
  return launch_mma(d, transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, ahi, alo, bhi, blo, sk,
                    partial_room, plan.sk_tiles, next_unit, gate, uplo, /*pdl=*/true);
}

// ---- panelled products ----------------------------------------------------

size_t wg_tc_product_workspace(const wg_device *d, int64_t m, int64_t k, const int64_t *widths, size_t count) {
  return product_layout(d->sm_count, m, k, widths, count).total;
}

namespace {
enum { EV_ENTRY = 0, EV_A_READY = 1, EV_PACKED = 2, EV_SLOT0 = 3, EV_SLOT1 = 4 };
}

wg_status wg_tc_product_begin(wg_tc_product *p, wg_device *d, int transA, int transB, int64_t m, int64_t k,
                              float alpha, const float *A, int64_t lda, float beta, const int64_t *widths,
                              size_t count, cudaEvent_t a_ready, const float *B0, int64_t ldb) {
  int64_t widest = 0;
  for (size_t i = 0; i < count; i++) widest = widths[i] > widest ? widths[i] : widest;
  const bool forced = d->sgemm_path >= WG_SGEMM_TF32X3_FUSED_BN256 && d->sgemm_path <= WG_SGEMM_TF32X3_PAIR;
  if (d->sgemm_path != WG_SGEMM_TF32X3_PACKED && widest > 0 &&
      (forced || (double)m * (double)widest * (double)k <= WG_FUSED_MAX_WORK) &&
      wg_tf32x3_fused_supported(d, transA, transB, m, widest, k, A, lda, B0, ldb)) {
    size_t bytes = 0;
    for (size_t i = 0; i < count; i++) {
      const size_t b = wg_tf32x3_fused_workspace(d, m, widths[i], k);
      bytes = b > bytes ? b : bytes;
    }
    void *ws = nullptr;
    wg_status st = wg_workspace(d, bytes, &ws);
    if (st != WG_OK) return st;
    *p = wg_tc_product{};
    p->d = d;
    p->transA = transA;
    p->transB = transB;
    p->m = m;
    p->k = k;
    p->alpha = alpha;
    p->beta = beta;
    p->A = A;
    p->lda = lda;
    p->ws = static_cast<char *>(ws);
    p->fused = true;
    p->ws_bytes = bytes;
    if (a_ready) WG_CUDA(cudaStreamWaitEvent(d->stream, a_ready, 0));
    d->stats.calls++;
    return WG_OK;
  }
  const ProductLayout P = product_layout(d->sm_count, m, k, widths, count);
  void *ws = nullptr;
  wg_status st = wg_workspace(d, P.total, &ws);
  if (st != WG_OK) return st;
  if (!d->side) WG_CUDA(cudaStreamCreateWithFlags(&d->side, cudaStreamNonBlocking));
  for (cudaEvent_t &e : d->tc_ev)
    if (!e) WG_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  p->d = d;
  p->transA = transA;
  p->transB = transB;
  p->m = m;
  p->k = k;
  p->alpha = alpha;
  p->beta = beta;
  p->A = A;
  p->lda = lda;
  p->ws = static_cast<char *>(ws);
  p->a_region = P.a_region;
  p->slot_bytes = P.slot_bytes;
  p->partial_room = P.partial_room;
  p->counter_room = P.counter_room;
  p->panels = 0;
  p->fused = false;
  p->ws_bytes = 0;
  // The splits run on the side stream after everything queued so far on the
  // device stream (earlier users of the workspace) and after op(A) is in place.
  WG_CUDA(cudaEventRecord(d->tc_ev[EV_ENTRY], d->stream));
  WG_CUDA(cudaStreamWaitEvent(d->side, d->tc_ev[EV_ENTRY], 0));
  if (a_ready) WG_CUDA(cudaStreamWaitEvent(d->side, a_ready, 0));
  p->epoch_a = wg_next_epoch(d);
  const Layout LA = layout_of(m, 1, k);
  float *ahi = reinterpret_cast<float *>(p->ws);
  float *alo = ahi + LA.a_bytes / sizeof(float);
  unsigned *counters = reinterpret_cast<unsigned *>(p->ws + P.a_region + 2 * P.slot_bytes + P.partial_room);
  st = launch_pack(d, d->side, pack_a_args(transA, A, lda, m, LA, ahi, alo, d->dwords + WG_DW_FALLBACK_A, p->epoch_a),
                   no_pack(), k, LA.kp, counters, P.counter_room, nullptr);
  if (st != WG_OK) return st;
  d->stats.calls++;
  return WG_OK;
}

wg_status wg_tc_product_panel(wg_tc_product *p, int64_t cols, const float *B, int64_t ldb, float *C, int64_t ldc,
                              cudaEvent_t b_ready) {
  wg_device *d = p->d;
  if (p->fused) {
    if (b_ready) WG_CUDA(cudaStreamWaitEvent(d->stream, b_ready, 0));
    wg_status st = wg_sgemm_tf32x3_fused(d, d->stream, p->transA, p->transB, p->m, cols, p->k, p->alpha, p->A, p->lda,
                                         B, ldb, p->beta, C, ldc, p->ws, p->ws_bytes);
    if (st != WG_OK) return st;
    d->stats.tf32x3_launches++;
    p->panels++;
    return WG_OK;
  }
  const int slot = (int)(p->panels & 1);
  const Layout L = layout_of(p->m, cols, p->k);
  float *ahi = reinterpret_cast<float *>(p->ws);
  float *alo = ahi + L.a_bytes / sizeof(float);
  float *bhi = reinterpret_cast<float *>(p->ws + p->a_region + (size_t)slot * p->slot_bytes);
  float *blo = bhi + L.b_bytes / sizeof(float);
  // Split buffer `slot` is free once the MMA two panels back has read it.
  if (p->panels >= 2) WG_CUDA(cudaStreamWaitEvent(d->side, d->tc_ev[EV_SLOT0 + slot], 0));
  if (b_ready) WG_CUDA(cudaStreamWaitEvent(d->side, b_ready, 0));
  unsigned *flag_b = d->dwords + WG_DW_FALLBACK_B0 + slot;
  const uint32_t epoch_b = wg_next_epoch(d);
  unsigned *next_unit = d->dwords + WG_DW_NEXT_UNIT0 + slot;
  wg_status st = launch_pack(d, d->side, no_pack(), pack_b_args(p->transB, B, ldb, cols, L, bhi, blo, flag_b, epoch_b),
                             p->k, L.kp, nullptr, 0, next_unit);
  if (st != WG_OK) return st;
  WG_CUDA(cudaEventRecord(d->tc_ev[EV_PACKED], d->side));
  WG_CUDA(cudaStreamWaitEvent(d->stream, d->tc_ev[EV_PACKED], 0));
  char *sk = p->ws + p->a_region + 2 * p->slot_bytes;
  const wg_gate gate{d->dwords + WG_DW_FALLBACK_A, flag_b, p->epoch_a, epoch_b};
  st = launch_mma(d, p->transA, p->transB, p->m, cols, p->k, p->alpha, p->A, p->lda, B, ldb, p->beta, C, ldc, ahi,
                  alo, bhi, blo, sk, p->partial_room, p->counter_room, next_unit, gate, WG_UPLO_FULL,
                  /*pdl=*/false);  // an event wait, not the split, precedes it on the stream
  if (st != WG_OK) return st;
  WG_CUDA(cudaEventRecord(d->tc_ev[EV_SLOT0 + slot], d->stream));
  d->stats.tf32x3_launches++;
  p->panels++;
  return WG_OK;
}

void wg_tc_product_join(wg_tc_product *p) {
  wg_device *d = p->d;
  if (!d || p->fused || !d->side) return;
  if (cudaEventRecord(d->tc_ev[EV_PACKED], d->side) == cudaSuccess)
    cudaStreamWaitEvent(d->stream, d->tc_ev[EV_PACKED], 0);
}
