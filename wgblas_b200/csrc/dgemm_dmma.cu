// dgemm on the FP64 tensor-core (DMMA) path: warp-level mma.sync .f64.
//
// tcgen05 has no f64 kind, so B200's FP64 tensor throughput is reached through
// the warp-level DMMA instruction. Two kernels share the warp tiling (a 128x128
// C tile per CTA, eight MMA warps as 2 (M) x 4 (N), each warp 64x32 = 4 x 4
// MMAs of 16x8, accumulators in registers):
//
// dgemm_tma_kernel (the main path) is fed by TMA. Thread 0 streams op(A) and
// op(B) k-slices (128 x 16 doubles each), STAGES - 1 ahead of the slice being
// multiplied, into a STAGES-deep shared-memory ring through three-dimensional
// tensor maps that reshape the operand so each
// warp's fragment load reads 32 consecutive doubles (no bank conflicts, no
// padding): an M- (or N-) contiguous operand is viewed as
// [rows/8][k][8] and a K-contiguous one as [k/4][rows][4]. Full / empty
// mbarriers replace the block-wide barrier of the register-staged kernel, so
// warps run ahead independently. After the k loop the accumulators are
// staged through shared memory and the epilogue reads old C and writes the
// new tile with 16-byte (double2) accesses, 32 lanes covering 512 contiguous
// bytes of a column. Every wait is clock-bounded: a stalled pipeline sets a
// bit in the device error word and the kernel returns.
//
// dgemm_regs_kernel (the fallback) stages tiles through registers with
// bounds-checked loads, so it takes any leading dimension and alignment; it
// runs when the tensor maps cannot describe the operands (odd leading
// dimensions, unaligned pointers, ragged edges that would make a tensor map
// read past the matrix).
//
// Fragment layouts (m16n8k8, f64; g = lane/4, t = lane%4):
//   A: a[v0 + 2*v1] = A(g + 8*v0, t + 4*v1)
//   B: b[v]         = B(t + 4*v, g)
//   C: c[v0 + 2*v1] = C(g + 8*v1, 2*t + v0)
// Each MMA sums its eight products inside the tensor core, so results are not
// bit-identical to a sequential FMA chain; they are held to the fp64 bound
// 4*K*2^-53*(|alpha||A||B| + |beta||C|). The epilogue is the reference's
// (src/shaders/sgemm_large.wgsl:303-304 as dgemm_small.wgsl:230-271 applies it)
// in fp64 with the beta term fused.
#include "internal.h"

namespace {

constexpr int BM = 128, BN = 128, BK = 16, NT = 256;
constexpr int PAD = 4;
constexpr int LDS_A = BM + PAD, LDS_B = BN + PAD;
constexpr int LPT = BM * BK / NT;  // 8 elements of each operand per thread per tile
constexpr size_t SMEM = sizeof(double) * 2 * BK * (LDS_A + LDS_B);

__device__ __forceinline__ void dmma_16x8x8(double (&d)[4], const double (&a)[4], const double (&b)[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f64.f64.f64.f64 "
      "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+d"(d[0]), "+d"(d[1]), "+d"(d[2]), "+d"(d[3])
      : "d"(a[0]), "d"(a[1]), "d"(a[2]), "d"(a[3]), "d"(b[0]), "d"(b[1]));
}

template <int TA, int TB>
__global__ void __launch_bounds__(NT, 1)
dgemm_regs_kernel(int64_t m, int64_t n, int64_t k, double alpha, const double *__restrict__ A, int64_t lda,
                  const double *__restrict__ B, int64_t ldb, double beta, double *__restrict__ C, int64_t ldc,
                  int uplo) {
  // gemmtr: a tile with no element in the triangle writes nothing (uniform exit, before any barrier).
  if (wg_tile_outside(uplo, (int64_t)blockIdx.x * BM, BM, (int64_t)blockIdx.y * BN, BN)) return;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  double *As = reinterpret_cast<double *>(smem_raw);  // [2][BK][LDS_A]
  double *Bs = As + 2 * BK * LDS_A;                  // [2][BK][LDS_B]

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int wm = (warp & 1) * 64, wn = (warp >> 1) * 32;
  const int64_t m0 = (int64_t)blockIdx.x * BM, n0 = (int64_t)blockIdx.y * BN;
  const int64_t ntiles = (k + BK - 1) / BK;

  double acc[4][4][4];
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int j = 0; j < 4; j++)
#pragma unroll
      for (int v = 0; v < 4; v++) acc[i][j][v] = 0.0;

  double ra[LPT], rb[LPT];
  auto load_tile = [&](int64_t tile) {
    const int64_t k0 = tile * BK;
#pragma unroll
    for (int q = 0; q < LPT; q++) {
      const int e = tid + q * NT;
      const int i = TA ? e / BK : e % BM;
      const int p = TA ? e % BK : e / BM;
      const int64_t gi = m0 + i, gp = k0 + p;
      ra[q] = (gi < m && gp < k) ? (TA ? A[gp + gi * lda] : A[gi + gp * lda]) : 0.0;
    }
#pragma unroll
    for (int q = 0; q < LPT; q++) {
      const int e = tid + q * NT;
      const int j = TB ? e % BN : e / BK;
      const int p = TB ? e / BN : e % BK;
      const int64_t gj = n0 + j, gp = k0 + p;
      rb[q] = (gj < n && gp < k) ? (TB ? B[gj + gp * ldb] : B[gp + gj * ldb]) : 0.0;
    }
  };
  auto store_tile = [&](int buf) {
    double *as = As + buf * BK * LDS_A;
    double *bs = Bs + buf * BK * LDS_B;
#pragma unroll
    for (int q = 0; q < LPT; q++) {
      const int e = tid + q * NT;
      const int i = TA ? e / BK : e % BM;
      const int p = TA ? e % BK : e / BM;
      as[p * LDS_A + i] = ra[q];
    }
#pragma unroll
    for (int q = 0; q < LPT; q++) {
      const int e = tid + q * NT;
      const int j = TB ? e % BN : e / BK;
      const int p = TB ? e / BN : e % BK;
      bs[p * LDS_B + j] = rb[q];
    }
  };

  if (ntiles > 0) {
    load_tile(0);
    store_tile(0);
    __syncthreads();
  }
  for (int64_t tile = 0; tile < ntiles; tile++) {
    const int cur = (int)(tile & 1);
    if (tile + 1 < ntiles) load_tile(tile + 1);
    const double *as = As + cur * BK * LDS_A;
    const double *bs = Bs + cur * BK * LDS_B;
#pragma unroll
    for (int ks = 0; ks < BK; ks += 8) {
      double a[4][4], b[4][2];
#pragma unroll
      for (int mt = 0; mt < 4; mt++) {
        const int r = wm + mt * 16 + g;
        a[mt][0] = as[(ks + t) * LDS_A + r];
        a[mt][1] = as[(ks + t) * LDS_A + r + 8];
        a[mt][2] = as[(ks + t + 4) * LDS_A + r];
        a[mt][3] = as[(ks + t + 4) * LDS_A + r + 8];
      }
#pragma unroll
      for (int nt = 0; nt < 4; nt++) {
        const int c = wn + nt * 8 + g;
        b[nt][0] = bs[(ks + t) * LDS_B + c];
        b[nt][1] = bs[(ks + t + 4) * LDS_B + c];
      }
#pragma unroll
      for (int mt = 0; mt < 4; mt++)
#pragma unroll
        for (int nt = 0; nt < 4; nt++) dmma_16x8x8(acc[mt][nt], a[mt], b[nt]);
    }
    if (tile + 1 < ntiles) store_tile(cur ^ 1);
    __syncthreads();
  }

  // The 16 old C values of one 16-row slice are loaded before any is written,
  // so the slice costs one memory round trip rather than one per element.
#pragma unroll
  for (int mt = 0; mt < 4; mt++) {
    double old[4][4];
#pragma unroll
    for (int nt = 0; nt < 4; nt++)
#pragma unroll
      for (int v = 0; v < 4; v++) {
        const int64_t row = m0 + wm + mt * 16 + g + 8 * (v >> 1);
        const int64_t col = n0 + wn + nt * 8 + 2 * t + (v & 1);
        old[nt][v] = (beta != 0.0 && row < m && col < n && wg_in_triangle(uplo, row, col)) ? C[row + col * ldc] : 0.0;
      }
#pragma unroll
    for (int nt = 0; nt < 4; nt++)
#pragma unroll
      for (int v = 0; v < 4; v++) {
        const int64_t row = m0 + wm + mt * 16 + g + 8 * (v >> 1);
        const int64_t col = n0 + wn + nt * 8 + 2 * t + (v & 1);
        if (row < m && col < n && wg_in_triangle(uplo, row, col)) {
          const double s = (alpha == 0.0) ? 0.0 : __dmul_rn(alpha, acc[mt][nt][v]);
          C[row + col * ldc] = (beta != 0.0) ? __fma_rn(beta, old[nt][v], s) : s;
        }
      }
  }
}

template <int TA, int TB>
cudaError_t launch_tt(cudaStream_t s, int64_t m, int64_t n, int64_t k, double alpha, const double *A, int64_t lda,
                      const double *B, int64_t ldb, double beta, double *C, int64_t ldc, int uplo) {
  auto kern = dgemm_regs_kernel<TA, TB>;
  cudaError_t e = wg_kernel_smem(kern, SMEM);
  if (e != cudaSuccess) return e;
  dim3 grid((unsigned)((m + BM - 1) / BM), (unsigned)((n + BN - 1) / BN));
  kern<<<grid, NT, SMEM, s>>>(m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, uplo);
  return cudaGetLastError();
}

}  // namespace


// ---- the TMA-fed kernel ---------------------------------------------------

#include "tcgen05.cuh"

namespace {

namespace tk {
constexpr int BM = 128, BN = 128, BK = 16, STAGES = 5;
constexpr int MMA_WARPS = 8, THREADS = 32 * MMA_WARPS;
constexpr int TILE = BM * BK * 8;  // bytes of one operand k-slice (BM == BN)
constexpr int STAGE = 2 * TILE;
constexpr int CS_LD = BM + 2;      // C staging tile: column-major, ld 130 doubles (conflict-free writes)
constexpr size_t RING = (size_t)STAGES * STAGE;
constexpr size_t SMEM = 128 /*alignment slack*/ + RING + 256 /*barriers*/;
constexpr long long WAIT_BUDGET = 4000000000LL;  // SM clocks (~2 s) before a wait gives up
static_assert((size_t)CS_LD * BN * 8 <= RING, "the C staging tile reuses the operand ring");
static_assert(BM == BN, "one tile size for both operands");

// Shared-memory offset (in doubles) of element (r, p) of a k-slice: r the row of
// op(A) (or column of op(B)) within the tile, p the k index within the slice.
// MN-contiguous operands land as [r/8][p][r%8], K-contiguous ones as [p/4][r][p%4].
template <bool KCONTIG>
__device__ __forceinline__ int slot(int r, int p) {
  return KCONTIG ? (p >> 2) * (BM * 4) + r * 4 + (p & 3) : (r >> 3) * (BK * 8) + p * 8 + (r & 7);
}
}  // namespace tk

__device__ __forceinline__ void mbar_arrive_cta(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(wgtc::smem_addr(bar)) : "memory");
}

struct TmaArgs {
  int64_t m, n, k;
  double alpha, beta;
  double *C;
  int64_t ldc;
  int uplo;
  int vec_ok;          // C and ldc allow 16-byte accesses
  unsigned *dwords;    // WG_DW_ERROR receives the wait-timeout bits
};

// TA: op(A) is K-contiguous (transA); TB: op(B) is K-contiguous (!transB).
template <int A_KCONTIG, int B_KCONTIG>
__global__ void __launch_bounds__(tk::THREADS, 1)
dgemm_tma_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                 const TmaArgs args) {
  constexpr int BM = tk::BM, BN = tk::BN, BK = tk::BK, STAGES = tk::STAGES, MMA_WARPS = tk::MMA_WARPS;
  constexpr int THREADS = tk::THREADS, TILE = tk::TILE, STAGE = tk::STAGE, CS_LD = tk::CS_LD;
  constexpr size_t RING = tk::RING;
  constexpr long long WAIT_BUDGET = tk::WAIT_BUDGET;
  using tk::slot;
  const int64_t m0 = (int64_t)blockIdx.x * BM, n0 = (int64_t)blockIdx.y * BN;
  if (wg_tile_outside(args.uplo, m0, BM, n0, BN)) return;  // gemmtr: uniform exit before any barrier

  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = smem_raw + ((128 - (wgtc::smem_addr(smem_raw) & 127)) & 127);
  uint64_t *full = reinterpret_cast<uint64_t *>(smem + RING);
  uint64_t *empty = full + STAGES;
  volatile int *abort_flag = reinterpret_cast<volatile int *>(empty + STAGES);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ntiles = (int)((args.k + BK - 1) / BK);
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      wgtc::mbar_init(&full[s], 1);
      wgtc::mbar_init(&empty[s], MMA_WARPS);
    }
    *abort_flag = 0;
    wgtc::fence_barrier_init();
  }
  __syncthreads();

  double acc[4][4][4];
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int j = 0; j < 4; j++)
#pragma unroll
      for (int v = 0; v < 4; v++) acc[i][j][v] = 0.0;

  // Thread 0 also feeds the ring: it issues the copies of k-slice `tile` into
  // stage tile % STAGES once every warp has released that stage (its empty
  // barrier), STAGES - 1 slices ahead of the slice being multiplied.
  int issued = 0;
  auto issue = [&](int tile) -> bool {
    const int s = tile % STAGES;
    if (!wgtc::mbar_wait_bounded(&empty[s], ((uint32_t)(tile / STAGES) & 1u) ^ 1u, WAIT_BUDGET)) return false;
    uint8_t *st = smem + (size_t)s * STAGE;
    wgtc::mbar_arrive_expect_tx(&full[s], STAGE);
    const int k0 = tile * BK;
    if (A_KCONTIG)
      wgtc::tma_load_3d(st, &map_a, &full[s], 0, (int)m0, k0 / 4);
    else
      wgtc::tma_load_3d(st, &map_a, &full[s], 0, k0, (int)(m0 / 8));
    if (B_KCONTIG)
      wgtc::tma_load_3d(st + TILE, &map_b, &full[s], 0, (int)n0, k0 / 4);
    else
      wgtc::tma_load_3d(st + TILE, &map_b, &full[s], 0, k0, (int)(n0 / 8));
    issued = tile + 1;
    return true;
  };
  if (threadIdx.x == 0) {
    wgtc::prefetch_tensormap(&map_a);
    wgtc::prefetch_tensormap(&map_b);
    for (int tile = 0; tile < STAGES - 1 && tile < ntiles; tile++) issue(tile);  // fresh stages: no wait
  }

  const int g = lane >> 2, t = lane & 3;
  const int wm = (warp & 1) * 64, wn = (warp >> 1) * 32;
  int kt = 0;
  for (; kt < ntiles; kt++) {
    if (threadIdx.x == 0 && kt + STAGES - 1 < ntiles && !*abort_flag && !issue(kt + STAGES - 1)) {
      atomicOr(args.dwords + WG_DW_ERROR, WG_DERR_TMA_WAIT);
      *abort_flag = 1;
    }
    const int s = kt % STAGES;
    const bool ok = wgtc::mbar_wait_bounded(&full[s], (uint32_t)(kt / STAGES) & 1u, WAIT_BUDGET);
    if (!__all_sync(0xffffffffu, ok && *abort_flag == 0)) {
      if (lane == 0 && !ok) atomicOr(args.dwords + WG_DW_ERROR, WG_DERR_TMA_WAIT);
      *abort_flag = 1;
      break;
    }
    const double *as = reinterpret_cast<const double *>(smem + (size_t)s * STAGE);
    const double *bs = as + TILE / 8;
#pragma unroll
    for (int ks = 0; ks < BK; ks += 8) {
      double a[4][4], b[4][2];
#pragma unroll
      for (int mt = 0; mt < 4; mt++) {
        const int r = wm + mt * 16 + g;
        a[mt][0] = as[slot<A_KCONTIG>(r, ks + t)];
        a[mt][1] = as[slot<A_KCONTIG>(r + 8, ks + t)];
        a[mt][2] = as[slot<A_KCONTIG>(r, ks + t + 4)];
        a[mt][3] = as[slot<A_KCONTIG>(r + 8, ks + t + 4)];
      }
#pragma unroll
      for (int nt = 0; nt < 4; nt++) {
        const int c = wn + nt * 8 + g;
        b[nt][0] = bs[slot<B_KCONTIG>(c, ks + t)];
        b[nt][1] = bs[slot<B_KCONTIG>(c, ks + t + 4)];
      }
#pragma unroll
      for (int mt = 0; mt < 4; mt++)
#pragma unroll
        for (int nt = 0; nt < 4; nt++) dmma_16x8x8(acc[mt][nt], a[mt], b[nt]);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive_cta(&empty[s]);  // this warp is done reading stage s
  }
  // After an abort, copies already issued may still be landing: wait for them
  // (bounded) before the CTA can exit and its shared memory be reused.
  if (threadIdx.x == 0)
    for (int q = kt; q < issued; q++)
      wgtc::mbar_wait_bounded(&full[q % STAGES], (uint32_t)(q / STAGES) & 1u, WAIT_BUDGET);

  // The ring is idle (every copy landed, every warp past its last stage): the
  // accumulators go through it as a column-major C tile.
  __syncthreads();
  if (*abort_flag) return;
  double *cs = reinterpret_cast<double *>(smem);
  {
#pragma unroll
    for (int mt = 0; mt < 4; mt++)
#pragma unroll
      for (int nt = 0; nt < 4; nt++)
#pragma unroll
        for (int v = 0; v < 4; v++) {
          const int r = wm + mt * 16 + g + 8 * (v >> 1);
          const int c = wn + nt * 8 + 2 * t + (v & 1);
          cs[c * CS_LD + r] = acc[mt][nt][v];
        }
  }
  __syncthreads();

  const double alpha = args.alpha, beta = args.beta;
  const int64_t m = args.m, n = args.n, ldc = args.ldc;
  double *C = args.C;
  const bool interior = m0 + BM <= m && n0 + BN <= n &&
                        (args.uplo == WG_UPLO_FULL || (args.uplo == WG_UPLO_LOWER ? n0 + BN - 1 <= m0
                                                                                  : n0 >= m0 + BM - 1));
  if (interior && args.vec_ok) {
    // 16-byte accesses: each thread handles two rows of one column per pass;
    // 64 threads cover a column, the 256 threads four columns at once.
    constexpr int PER_PASS = THREADS / 64;  // columns per pass
    const int tid = threadIdx.x;
    if (tid < 64 * PER_PASS) {
      const int r = 2 * (tid & 63);
      for (int c0 = tid >> 6; c0 < BN; c0 += 4 * PER_PASS) {
        double2 old[4];
        if (beta != 0.0) {
#pragma unroll
          for (int q = 0; q < 4; q++)
            old[q] = *reinterpret_cast<const double2 *>(C + (m0 + r) + (n0 + c0 + q * PER_PASS) * ldc);
        }
#pragma unroll
        for (int q = 0; q < 4; q++) {
          const int c = c0 + q * PER_PASS;
          const double2 v = *reinterpret_cast<const double2 *>(cs + c * CS_LD + r);
          double2 o;
          o.x = (alpha == 0.0) ? 0.0 : __dmul_rn(alpha, v.x);
          o.y = (alpha == 0.0) ? 0.0 : __dmul_rn(alpha, v.y);
          if (beta != 0.0) {
            o.x = __fma_rn(beta, old[q].x, o.x);
            o.y = __fma_rn(beta, old[q].y, o.y);
          }
          *reinterpret_cast<double2 *>(C + (m0 + r) + (n0 + c) * ldc) = o;
        }
      }
    }
  } else {
    // Edge or diagonal tiles, or C not 16-byte aligned: one element per thread
    // per pass, a warp covering 32 consecutive rows of a column.
    for (int e = threadIdx.x; e < BM * BN; e += THREADS) {
      const int r = e % BM, c = e / BM;
      const int64_t row = m0 + r, col = n0 + c;
      if (row < m && col < n && wg_in_triangle(args.uplo, row, col)) {
        const double s = (alpha == 0.0) ? 0.0 : __dmul_rn(alpha, cs[c * CS_LD + r]);
        C[row + col * ldc] = (beta != 0.0) ? __fma_rn(beta, C[row + col * ldc], s) : s;
      }
    }
  }
}

// Tensor map of one operand as the kernel's k-slices see it (see slot()).
// rows = m (op(A)) or n (op(B)); ld the operand's leading dimension. Returns
// false when the layout cannot be described (the caller then uses the
// register-staged kernel).
bool make_dmap(CUtensorMap *map, const double *ptr, bool kcontig, int64_t rows, int64_t k, int64_t ld) {
  wg_encode_tiled_fn fn = wg_encode_tiled();
  if (!fn) return false;
  if (reinterpret_cast<uintptr_t>(ptr) % 16 != 0 || ld % 2 != 0) return false;
  cuuint64_t dims[3], strides[2];
  cuuint32_t box[3];
  if (kcontig) {
    // element (r, p) at ptr[p + r*ld]: [k/4][rows][4], read whole groups of 4 in k
    if (k % 4 != 0) return false;
    dims[0] = 4; dims[1] = (cuuint64_t)rows; dims[2] = (cuuint64_t)(k / 4);
    strides[0] = (cuuint64_t)ld * 8; strides[1] = 32;
    box[0] = 4; box[1] = tk::BM; box[2] = tk::BK / 4;
  } else {
    // element (r, p) at ptr[r + p*ld]: [rows/8][k][8], read whole groups of 8 rows
    if (rows % 8 != 0) return false;
    dims[0] = 8; dims[1] = (cuuint64_t)k; dims[2] = (cuuint64_t)(rows / 8);
    strides[0] = (cuuint64_t)ld * 8; strides[1] = 64;
    box[0] = 8; box[1] = tk::BK; box[2] = tk::BM / 8;
  }
  if (dims[1] >= ((cuuint64_t)1 << 31) || dims[2] >= ((cuuint64_t)1 << 31) || strides[0] >= ((cuuint64_t)1 << 40))
    return false;
  cuuint32_t estr[3] = {1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT64, 3, const_cast<double *>(ptr), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int AK, int BKC>
cudaError_t launch_tma(cudaStream_t s, const CUtensorMap &ma, const CUtensorMap &mb, const TmaArgs &args) {
  auto kern = dgemm_tma_kernel<AK, BKC>;
  cudaError_t e = wg_kernel_smem(kern, tk::SMEM);
  if (e != cudaSuccess) return e;
  dim3 grid((unsigned)((args.m + tk::BM - 1) / tk::BM), (unsigned)((args.n + tk::BN - 1) / tk::BN));
  kern<<<grid, tk::THREADS, tk::SMEM, s>>>(ma, mb, args);
  return cudaGetLastError();
}

}  // namespace

wg_status wg_dgemm_dmma(wg_device *d, int transA, int transB, int64_t m, int64_t n, int64_t k, double alpha,
                        const double *A, int64_t lda, const double *B, int64_t ldb, double beta, double *C,
                        int64_t ldc, int uplo) {
  if ((n + tk::BN - 1) / tk::BN > 65535)
    return wg_fail(WG_ERR_NOT_SUPPORTED, "dgemm: n=%lld exceeds the tile grid", (long long)n);
  cudaStream_t s = d->stream;
  const bool a_k = transA != 0, b_k = transB == 0;
  CUtensorMap ma, mb;
  if (make_dmap(&ma, A, a_k, m, k, lda) && make_dmap(&mb, B, b_k, n, k, ldb)) {
    const TmaArgs args{m, n, k, alpha, beta, C, ldc, uplo,
                       (reinterpret_cast<uintptr_t>(C) % 16 == 0 && ldc % 2 == 0) ? 1 : 0, d->dwords};
    wg_launch_scope scope(d, "dgemm_dmma");
    cudaError_t e = a_k ? (b_k ? launch_tma<1, 1>(s, ma, mb, args) : launch_tma<1, 0>(s, ma, mb, args))
                        : (b_k ? launch_tma<0, 1>(s, ma, mb, args) : launch_tma<0, 0>(s, ma, mb, args));
    WG_CUDA(e);
    return WG_OK;
  }
  wg_launch_scope scope(d, "dgemm_dmma_regs");
  cudaError_t e = transA ? (transB ? launch_tt<1, 1>(s, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, uplo)
                                   : launch_tt<1, 0>(s, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, uplo))
                         : (transB ? launch_tt<0, 1>(s, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, uplo)
                                   : launch_tt<0, 0>(s, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, uplo));
  WG_CUDA(e);
  return WG_OK;
}
