// The FFMA / DFMA tile of the SIMT GEMM: 128x128 tiles of C, 256 threads,
// each element one sequential fused multiply-add chain over p = 0..k-1 and
// then the reference's epilogue (src/shaders/sgemm_large.wgsl:299-304, the beta
// term fused). Shared by the SIMT kernel (gemm_simt.cu) and by the 3xTF32 MMA
// kernel's fallback (sgemm_tf32x3.cu), which computes C itself when the split
// ruled its operands out, so both give the same bits.
#pragma once

#include "internal.h"

namespace wgsimt {

template <typename T>
__device__ __forceinline__ T fma_rn(T a, T b, T c);
template <>
__device__ __forceinline__ float fma_rn<float>(float a, float b, float c) { return __fmaf_rn(a, b, c); }
template <>
__device__ __forceinline__ double fma_rn<double>(double a, double b, double c) { return __fma_rn(a, b, c); }
template <typename T>
__device__ __forceinline__ T mul_rn(T a, T b);
template <>
__device__ __forceinline__ float mul_rn<float>(float a, float b) { return __fmul_rn(a, b); }
template <>
__device__ __forceinline__ double mul_rn<double>(double a, double b) { return __dmul_rn(a, b); }

// Epilogue of one element (sgemm_large.wgsl:303-304, with the beta term fused).
template <typename T>
__device__ __forceinline__ T epilogue(T acc, T alpha, T beta, T c_old) {
  T s = (alpha == T(0)) ? T(0) : mul_rn(alpha, acc);
  return (beta != T(0)) ? fma_rn(beta, c_old, s) : s;
}

// Four consecutive elements through 16-byte vectors (one float4 or two double2).
template <typename T>
struct Vec4;
template <>
struct Vec4<float> {
  __device__ __forceinline__ static void load(float *d, const float *s) {
    float4 v = *reinterpret_cast<const float4 *>(s);
    d[0] = v.x; d[1] = v.y; d[2] = v.z; d[3] = v.w;
  }
  __device__ __forceinline__ static void store(float *d, const float *s) {
    *reinterpret_cast<float4 *>(d) = make_float4(s[0], s[1], s[2], s[3]);
  }
};
template <>
struct Vec4<double> {
  __device__ __forceinline__ static void load(double *d, const double *s) {
    double2 v0 = reinterpret_cast<const double2 *>(s)[0];
    double2 v1 = reinterpret_cast<const double2 *>(s)[1];
    d[0] = v0.x; d[1] = v0.y; d[2] = v1.x; d[3] = v1.y;
  }
  __device__ __forceinline__ static void store(double *d, const double *s) {
    reinterpret_cast<double2 *>(d)[0] = make_double2(s[0], s[1]);
    reinterpret_cast<double2 *>(d)[1] = make_double2(s[2], s[3]);
  }
};

constexpr int BM = 128, BN = 128, BK = 8, TM = 8, TN = 8;
constexpr int TX = BM / TM, TY = BN / TN, NT = TX * TY;  // 16 x 16 = 256 threads
constexpr int LPT_A = BM * BK / NT, LPT_B = BK * BN / NT;  // 4 elements each

template <typename T>
constexpr int pad() { return 16 / (int)sizeof(T); }
template <typename T>
constexpr int lda_s() { return BM + pad<T>(); }  // shared row stride of the A tile
template <typename T>
constexpr int ldb_s() { return BN + pad<T>(); }
template <typename T>
constexpr size_t smem_bytes() { return sizeof(T) * 2 * BK * (lda_s<T>() + ldb_s<T>()); }

// One tile at (m0, n0): every one of the block's NT threads calls it; As and Bs
// are 2*BK*lda_s<T>() and 2*BK*ldb_s<T>() elements of shared memory. kk = 0
// reads neither A nor B (alpha == 0). With mask.flags set, only columns of
// flagged tiles are written.
template <typename T, int TA, int TB>
__device__ __forceinline__ void tile(int64_t m0, int64_t n0, int64_t m, int64_t n, int64_t kk, T alpha,
                                     const T *__restrict__ A, int64_t lda, const T *__restrict__ B, int64_t ldb,
                                     T beta, T *__restrict__ C, int64_t ldc, const wg_tile_mask &mask, int uplo,
                                     T *As, T *Bs) {
  const int tid = threadIdx.x;
  const int tx = tid % TX, ty = tid / TX;
  const int64_t ntiles = (kk + BK - 1) / BK;
  __syncthreads();  // the previous tile's last reads of shared memory are done

  T acc[TM][TN];
#pragma unroll
  for (int i = 0; i < TM; i++)
#pragma unroll
    for (int j = 0; j < TN; j++) acc[i][j] = T(0);

  T ra[LPT_A], rb[LPT_B];
  auto load_tile = [&](int64_t t) {
    const int64_t k0 = t * BK;
#pragma unroll
    for (int q = 0; q < LPT_A; q++) {
      const int e = tid + q * NT;
      const int i = TA ? e / BK : e % BM;
      const int p = TA ? e % BK : e / BM;
      const int64_t gi = m0 + i, gp = k0 + p;
      ra[q] = (gi < m && gp < kk) ? (TA ? A[gp + gi * lda] : A[gi + gp * lda]) : T(0);
    }
#pragma unroll
    for (int q = 0; q < LPT_B; q++) {
      const int e = tid + q * NT;
      const int j = TB ? e % BN : e / BK;
      const int p = TB ? e / BN : e % BK;
      const int64_t gj = n0 + j, gp = k0 + p;
      rb[q] = (gj < n && gp < kk) ? (TB ? B[gj + gp * ldb] : B[gp + gj * ldb]) : T(0);
    }
  };
  auto store_tile = [&](int buf) {
    T *as = As + buf * BK * lda_s<T>();
    T *bs = Bs + buf * BK * ldb_s<T>();
#pragma unroll
    for (int q = 0; q < LPT_A; q++) {
      const int e = tid + q * NT;
      const int i = TA ? e / BK : e % BM;
      const int p = TA ? e % BK : e / BM;
      as[p * lda_s<T>() + i] = ra[q];
    }
#pragma unroll
    for (int q = 0; q < LPT_B; q++) {
      const int e = tid + q * NT;
      const int j = TB ? e % BN : e / BK;
      const int p = TB ? e / BN : e % BK;
      bs[p * ldb_s<T>() + j] = rb[q];
    }
  };

  if (ntiles > 0) {
    load_tile(0);
    store_tile(0);
    __syncthreads();
  }
  for (int64_t t = 0; t < ntiles; t++) {
    const int cur = (int)(t & 1);
    if (t + 1 < ntiles) load_tile(t + 1);
    const T *as = As + cur * BK * lda_s<T>();
    const T *bs = Bs + cur * BK * ldb_s<T>();
#pragma unroll
    for (int p = 0; p < BK; p++) {
      T a[TM], b[TN];
      Vec4<T>::load(a, as + p * lda_s<T>() + 4 * tx);
      Vec4<T>::load(a + 4, as + p * lda_s<T>() + BM / 2 + 4 * tx);
      Vec4<T>::load(b, bs + p * ldb_s<T>() + 4 * ty);
      Vec4<T>::load(b + 4, bs + p * ldb_s<T>() + BN / 2 + 4 * ty);
#pragma unroll
      for (int i = 0; i < TM; i++)
#pragma unroll
        for (int j = 0; j < TN; j++) acc[i][j] = fma_rn(a[i], b[j], acc[i][j]);
    }
    if (t + 1 < ntiles) store_tile(cur ^ 1);
    __syncthreads();
  }

  // Epilogue: columns j, runs of four rows along m.
#pragma unroll
  for (int g = 0; g < 2; g++)
#pragma unroll
    for (int r = 0; r < 4; r++) {
      const int64_t gj = n0 + g * (BN / 2) + 4 * ty + r;
      if (gj >= n) continue;
      if (mask.flags && mask.flags[m0 / BM + (gj / mask.bn) * mask.tiles_m] != mask.epoch) continue;
#pragma unroll
      for (int h = 0; h < 2; h++) {
        const int64_t gi = m0 + h * (BM / 2) + 4 * tx;
        if (gi >= m) continue;
        T *cp = C + gi + gj * ldc;
        T v[4], old[4] = {T(0), T(0), T(0), T(0)};
        const bool full = gi + 3 < m && (reinterpret_cast<uintptr_t>(cp) % 16 == 0) &&
                          wg_in_triangle(uplo, gi, gj) && wg_in_triangle(uplo, gi + 3, gj);
        if (full) {
          if (beta != T(0)) Vec4<T>::load(old, cp);
#pragma unroll
          for (int q = 0; q < 4; q++) v[q] = epilogue(acc[h * 4 + q][g * 4 + r], alpha, beta, old[q]);
          Vec4<T>::store(cp, v);
        } else {
#pragma unroll
          for (int q = 0; q < 4; q++)
            if (gi + q < m && wg_in_triangle(uplo, gi + q, gj)) {
              T o = (beta != T(0)) ? cp[q] : T(0);
              cp[q] = epilogue(acc[h * 4 + q][g * 4 + r], alpha, beta, o);
            }
        }
      }
    }
}

}  // namespace wgsimt
