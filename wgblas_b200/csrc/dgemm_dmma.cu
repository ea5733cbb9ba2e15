// dgemm on the FP64 tensor-core (DMMA) path: mma.sync.m16n8k8 .f64.
//
// tcgen05 has no f64 kind, so B200's FP64 tensor throughput is reached through
// the warp-level DMMA instruction. A 128x128 C tile per 256-thread CTA, eight
// warps as 2 (M) x 4 (N), each warp 64x32 = 4 x 4 MMAs of 16x8 per 8-deep k
// step, accumulators in registers. op(A) and op(B) tiles (128 x 16 and 16 x 128)
// are staged m- and n-contiguous in double-buffered shared memory through
// registers with bounds-checked loads, so every transpose pair, leading
// dimension and alignment is handled; the next tile's global loads are in
// flight while the current one is multiplied. Rows of the shared tiles are
// padded by four doubles, which puts the four k rows a fragment load touches
// on disjoint banks.
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
dgemm_dmma_kernel(int64_t m, int64_t n, int64_t k, double alpha, const double *__restrict__ A, int64_t lda,
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
  auto kern = dgemm_dmma_kernel<TA, TB>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM);
  if (e != cudaSuccess) return e;
  dim3 grid((unsigned)((m + BM - 1) / BM), (unsigned)((n + BN - 1) / BN));
  kern<<<grid, NT, SMEM, s>>>(m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, uplo);
  return cudaGetLastError();
}

}  // namespace

cudaError_t wg_launch_dgemm_dmma(cudaStream_t s, int transA, int transB, int64_t m, int64_t n, int64_t k,
                                 double alpha, const double *A, int64_t lda, const double *B, int64_t ldb,
                                 double beta, double *C, int64_t ldc, int uplo) {
  if ((n + BN - 1) / BN > 65535) return cudaErrorInvalidConfiguration;
  if (transA)
    return transB ? launch_tt<1, 1>(s, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, uplo)
                  : launch_tt<1, 0>(s, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, uplo);
  return transB ? launch_tt<0, 1>(s, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, uplo)
                : launch_tt<0, 0>(s, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, uplo);
}
