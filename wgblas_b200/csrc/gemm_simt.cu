// Register-blocked SIMT GEMM on the FP32 (FFMA) and FP64 (DFMA) pipes.
//
// It handles every transpose combination, any leading dimension and any
// alignment, and is the path for shapes and operands the tensor-core kernel
// does not take (see gemm.cu). Each output element is one sequential fused
// multiply-add chain over p = 0..k-1, followed by the reference's epilogue
// (src/shaders/sgemm_large.wgsl:299-304):
//   s = (alpha == 0) ? 0 : alpha*acc;   C = (beta != 0) ? fma(beta, C, s) : s
// which is also the arithmetic the CPU oracle's FMA restatement performs, so the
// two agree bit for bit.
//
// Layout: a 128x128 C tile per 256-thread CTA; thread (tx, ty) owns rows
// {h*64 + 4*tx + q} and columns {g*64 + 4*ty + r} (h, g in {0,1}; q, r < 4), so a
// warp's stores along m are contiguous. Tiles of op(A) (128 x 8) and op(B)
// (8 x 128) are staged m- and n-contiguous in double-buffered shared memory
// through registers; the next tile's global loads are in flight while the
// current one is multiplied.
#include "internal.h"

namespace {

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
constexpr int64_t GATED_GRID = 148;  // one wave on a B200: a closed gate costs one CTA launch per SM
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

template <typename T, int TA, int TB>
__global__ void __launch_bounds__(NT, 1)
gemm_simt_kernel(int64_t m, int64_t n, int64_t k, T alpha, const T *__restrict__ A, int64_t lda,
                 const T *__restrict__ B, int64_t ldb, T beta, T *__restrict__ C, int64_t ldc,
                 unsigned *dwords, wg_gate gate, int gated, wg_tile_mask mask, int uplo) {
  if (gated) {
    // Device-side fallback of the 3xTF32 path: run only if its operand check failed.
    if (!wg_gate_open(gate)) return;
    if (blockIdx.x == 0 && threadIdx.x == 0) atomicAdd(dwords + WG_DW_FALLBACKS, 1u);
  }
  extern __shared__ __align__(16) unsigned char smem_raw[];
  T *As = reinterpret_cast<T *>(smem_raw);       // [2][BK][lda_s]
  T *Bs = As + 2 * BK * lda_s<T>();             // [2][BK][ldb_s]

  const int tid = threadIdx.x;
  const int tx = tid % TX, ty = tid / TX;
  const int64_t kk = (alpha == T(0)) ? 0 : k;  // alpha == 0 reads neither A nor B
  const int64_t ntiles = (kk + BK - 1) / BK;
  const int64_t tiles_m = (m + BM - 1) / BM, tiles = tiles_m * ((n + BN - 1) / BN);
  // Tiles in column order of C (m fastest); the grid strides over them, so a gated
  // launch needs only a few CTAs to exit when its gate is closed.
  for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
  const int64_t m0 = (tile % tiles_m) * BM, n0 = (tile / tiles_m) * BN;
  // gemmtr: a tile with no element in the triangle writes nothing (uniform skip).
  if (wg_tile_outside(uplo, m0, BM, n0, BN)) continue;
  // Masked (the fallback of a fused 3xTF32 call): only columns of flagged tiles.
  if (mask.flags) {
    const int64_t ftm = m0 / BM, last = (n0 + BN < n ? n0 + BN : n) - 1;
    bool any = false;
    for (int64_t ftn = n0 / mask.bn; ftn <= last / mask.bn; ftn++)
      any |= mask.flags[ftm + ftn * mask.tiles_m] == mask.epoch;
    if (!any) continue;
  }
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
}

// C = epilogue(0) elementwise: the k == 0 and alpha == 0 cases.
template <typename T>
__global__ void scale_kernel(int64_t m, int64_t n, T alpha, T beta, T *__restrict__ C, int64_t ldc, int uplo) {
  const int64_t total = m * n;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = e % m, j = e / m;
    if (!wg_in_triangle(uplo, i, j)) continue;
    T *cp = C + i + j * ldc;
    const T old = (beta != T(0)) ? *cp : T(0);
    *cp = epilogue(T(0), alpha, beta, old);
  }
}

template <typename T, int TA, int TB>
cudaError_t launch_tt(cudaStream_t s, int64_t m, int64_t n, int64_t k, T alpha, const T *A,
                      int64_t lda, const T *B, int64_t ldb, T beta, T *C, int64_t ldc,
                      unsigned *dwords, const wg_gate *gate, const wg_tile_mask *mask, int uplo) {
  auto kern = gemm_simt_kernel<T, TA, TB>;
  // Per-device attribute: set on every launch so each device that runs the kernel has it.
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem_bytes<T>());
  // The same shared-memory carveout as the tensor-core kernels it follows, so an
  // SM need not reconfigure between them.
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
  if (e != cudaSuccess) return e;
  // One CTA per tile; a gated launch (usually a no-op) strides with at most one
  // CTA per SM of a B200, so its closed-gate exit costs little more than the launch.
  int64_t grid = ((m + BM - 1) / BM) * ((n + BN - 1) / BN);
  if (gate && grid > GATED_GRID) grid = GATED_GRID;
  const wg_gate g = gate ? *gate : wg_gate{nullptr, nullptr, 0u, 0u};
  const wg_tile_mask mk = mask ? *mask : wg_tile_mask{nullptr, 1, 1, 0u};
  kern<<<(unsigned)grid, NT, smem_bytes<T>(), s>>>(m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, dwords, g,
                                                   gate ? 1 : 0, mk, uplo);
  return cudaGetLastError();
}

}  // namespace

template <typename T>
cudaError_t wg_launch_gemm_simt_masked(cudaStream_t s, int transA, int transB, int64_t m, int64_t n, int64_t k,
                                       T alpha, const T *A, int64_t lda, const T *B, int64_t ldb, T beta, T *C,
                                       int64_t ldc, unsigned *dwords, const wg_gate *gate, const wg_tile_mask *mask,
                                       int uplo) {
  if (((m + BM - 1) / BM) * ((n + BN - 1) / BN) >= ((int64_t)1 << 31)) return cudaErrorInvalidConfiguration;
  if (transA) {
    return transB ? launch_tt<T, 1, 1>(s, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, dwords, gate, mask, uplo)
                  : launch_tt<T, 1, 0>(s, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, dwords, gate, mask, uplo);
  }
  return transB ? launch_tt<T, 0, 1>(s, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, dwords, gate, mask, uplo)
                : launch_tt<T, 0, 0>(s, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, dwords, gate, mask, uplo);
}

template <typename T>
cudaError_t wg_launch_gemm_simt(cudaStream_t s, int transA, int transB, int64_t m, int64_t n,
                                int64_t k, T alpha, const T *A, int64_t lda, const T *B,
                                int64_t ldb, T beta, T *C, int64_t ldc, unsigned *dwords,
                                const wg_gate *gate, int uplo) {
  return wg_launch_gemm_simt_masked<T>(s, transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, dwords,
                                       gate, nullptr, uplo);
}

template <typename T>
cudaError_t wg_launch_scale(cudaStream_t s, int64_t m, int64_t n, T alpha, T beta, T *C, int64_t ldc, int uplo) {
  const int64_t total = m * n;
  int64_t blocks = (total + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  if (blocks < 1) blocks = 1;
  scale_kernel<T><<<(unsigned)blocks, 256, 0, s>>>(m, n, alpha, beta, C, ldc, uplo);
  return cudaGetLastError();
}

template cudaError_t wg_launch_gemm_simt<float>(cudaStream_t, int, int, int64_t, int64_t, int64_t, float,
                                                const float *, int64_t, const float *, int64_t, float,
                                                float *, int64_t, unsigned *, const wg_gate *, int);
template cudaError_t wg_launch_gemm_simt<double>(cudaStream_t, int, int, int64_t, int64_t, int64_t, double,
                                                 const double *, int64_t, const double *, int64_t, double,
                                                 double *, int64_t, unsigned *, const wg_gate *, int);
template cudaError_t wg_launch_gemm_simt_masked<float>(cudaStream_t, int, int, int64_t, int64_t, int64_t, float,
                                                       const float *, int64_t, const float *, int64_t, float,
                                                       float *, int64_t, unsigned *, const wg_gate *,
                                                       const wg_tile_mask *, int);
template cudaError_t wg_launch_scale<float>(cudaStream_t, int64_t, int64_t, float, float, float *, int64_t, int);
template cudaError_t wg_launch_scale<double>(cudaStream_t, int64_t, int64_t, double, double, double *, int64_t, int);
