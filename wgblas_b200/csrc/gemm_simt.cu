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
#include "simt_tile.cuh"

namespace {

using namespace wgsimt;

constexpr int64_t GATED_GRID = 148;  // one wave on a B200: a closed gate costs one CTA launch per SM

template <typename T, int TA, int TB>
__global__ void __launch_bounds__(NT, 1)
gemm_simt_kernel(int64_t m, int64_t n, int64_t k, T alpha, const T *__restrict__ A, int64_t lda,
                 const T *__restrict__ B, int64_t ldb, T beta, T *__restrict__ C, int64_t ldc,
                 unsigned *dwords, wg_gate gate, int gated, wg_tile_mask mask, int uplo) {
  if (gated) {
    // Device-side fallback of the 3xTF32 path: run only if its operand check
    // failed. Launched programmatically, it may be resident before the kernel
    // that sets the gate has finished: wait for that kernel first.
    wg_pdl_wait();
    if (!wg_gate_open(gate)) return;
    if (blockIdx.x == 0 && threadIdx.x == 0) atomicAdd(dwords + WG_DW_FALLBACKS, 1u);
  }
  extern __shared__ __align__(16) unsigned char smem_raw[];
  T *As = reinterpret_cast<T *>(smem_raw);       // [2][BK][lda_s]
  T *Bs = As + 2 * BK * lda_s<T>();             // [2][BK][ldb_s]

  const int64_t kk = (alpha == T(0)) ? 0 : k;  // alpha == 0 reads neither A nor B
  const int64_t tiles_m = (m + BM - 1) / BM, tiles = tiles_m * ((n + BN - 1) / BN);
  // Tiles in column order of C (m fastest); the grid strides over them, so a gated
  // launch needs only a few CTAs to exit when its gate is closed.
  for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x) {
    const int64_t m0 = (t % tiles_m) * BM, n0 = (t / tiles_m) * BN;
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
    tile<T, TA, TB>(m0, n0, m, n, kk, alpha, A, lda, B, ldb, beta, C, ldc, mask, uplo, As, Bs);
  }
}

// ---- small products ---------------------------------------------------------
// The same per-element arithmetic (one FMA chain over p = 0..k-1 in order, then
// the epilogue) on 32 x 64 tiles of C, so that a product of a few hundred rows
// and columns still spreads over every SM: 128 threads, each owning 4 rows x 4
// columns (thread (tx, ty) = (tid % 8, tid / 8): a warp covers 8 x 4 threads,
// so each of its 16-byte shared-memory reads of A and of B is one wavefront).
// Tiles of op(A) (32 x 16) and op(B) (16 x 64) stream through an S_STAGES-deep
// ring with 4-byte cp.async (zero-filled past the edges; any transpose, leading
// dimension and alignment), so several k-tiles are in flight while one is
// multiplied. The last k-tile runs only its real p: no padded term is added.
constexpr int S_BM = 32, S_BN = 64, S_BK = 16, S_STAGES = 6, S_NT = 128;
constexpr int S_LDA = S_BM + 4, S_LDB = S_BN + 4;  // shared row strides (floats)
constexpr int S_STAGE = S_BK * (S_LDA + S_LDB);
constexpr size_t S_SMEM = sizeof(float) * S_STAGES * S_STAGE;

__device__ __forceinline__ void cp_async4(float *dst, const float *src, bool pred) {
  // src-size 0 writes a zero and reads nothing.
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src), "r"(pred ? 4 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

template <int TA, int TB>
__global__ void __launch_bounds__(S_NT, 4)
gemm_simt_small_kernel(int64_t m, int64_t n, int64_t k, float alpha, const float *__restrict__ A, int64_t lda,
                       const float *__restrict__ B, int64_t ldb, float beta, float *__restrict__ C, int64_t ldc,
                       int uplo) {
  extern __shared__ __align__(16) float sm[];
  const int tid = threadIdx.x, tx = tid % 8, ty = tid / 8;
  const int64_t tiles_m = (m + S_BM - 1) / S_BM;
  const int64_t m0 = (blockIdx.x % tiles_m) * S_BM, n0 = (blockIdx.x / tiles_m) * S_BN;
  if (wg_tile_outside(uplo, m0, S_BM, n0, S_BN)) return;
  const int64_t kk = (alpha == 0.0f) ? 0 : k;  // alpha == 0 reads neither A nor B
  const int64_t ntiles = (kk + S_BK - 1) / S_BK;

  // Stage t of the ring: op(A) at [p][i], op(B) at [p][j]. Consecutive threads
  // read consecutive addresses of whichever dimension the operand stores contiguously.
  auto issue = [&](int64_t t) {
    float *as = sm + (t % S_STAGES) * S_STAGE, *bs = as + S_BK * S_LDA;
    const int64_t k0 = t * S_BK;
#pragma unroll
    for (int q = 0; q < S_BM * S_BK / S_NT; q++) {
      const int e = tid + q * S_NT;
      const int i = TA ? e / S_BK : e % S_BM, p = TA ? e % S_BK : e / S_BM;
      const int64_t gi = m0 + i, gp = k0 + p;
      const bool in = gi < m && gp < kk;
      cp_async4(as + p * S_LDA + i, in ? (TA ? A + gp + gi * lda : A + gi + gp * lda) : A, in);
    }
#pragma unroll
    for (int q = 0; q < S_BN * S_BK / S_NT; q++) {
      const int e = tid + q * S_NT;
      const int j = TB ? e % S_BN : e / S_BK, p = TB ? e / S_BN : e % S_BK;
      const int64_t gj = n0 + j, gp = k0 + p;
      const bool in = gj < n && gp < kk;
      cp_async4(bs + p * S_LDB + j, in ? (TB ? B + gj + gp * ldb : B + gp + gj * ldb) : B, in);
    }
  };

  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int j = 0; j < 4; j++) acc[i][j] = 0.0f;

#pragma unroll
  for (int s = 0; s < S_STAGES - 1; s++) {
    if (s < ntiles) issue(s);
    cp_async_commit();  // one group per stage, empty ones included, so the wait count below holds
  }
  for (int64_t t = 0; t < ntiles; t++) {
    cp_async_wait<S_STAGES - 2>();  // this thread's copies of tile t have landed
    __syncthreads();                // everyone's have, and tile t-1's buffer is free
    if (t + S_STAGES - 1 < ntiles) issue(t + S_STAGES - 1);
    cp_async_commit();
    const float *as = sm + (t % S_STAGES) * S_STAGE, *bs = as + S_BK * S_LDA;
    const int64_t rem = kk - t * S_BK;
    auto step = [&](int p) {
      float a[4], b[4];
      Vec4<float>::load(a, as + p * S_LDA + 4 * tx);
      Vec4<float>::load(b, bs + p * S_LDB + 4 * ty);
#pragma unroll
      for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = __fmaf_rn(a[i], b[j], acc[i][j]);
    };
    if (rem >= S_BK) {
#pragma unroll
      for (int p = 0; p < S_BK; p++) step(p);
    } else {
      for (int p = 0; p < (int)rem; p++) step(p);
    }
  }
  cp_async_wait<0>();

  // Epilogue: four rows along m per column, 16-byte stores where they fit.
  const int64_t gi = m0 + 4 * tx;
  if (gi >= m) return;
#pragma unroll
  for (int r = 0; r < 4; r++) {
    const int64_t gj = n0 + 4 * ty + r;
    if (gj >= n) continue;
    float *cp = C + gi + gj * ldc;
    const bool full = gi + 3 < m && (reinterpret_cast<uintptr_t>(cp) % 16 == 0) && wg_in_triangle(uplo, gi, gj) &&
                      wg_in_triangle(uplo, gi + 3, gj);
    if (full) {
      float v[4], old[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      if (beta != 0.0f) Vec4<float>::load(old, cp);
#pragma unroll
      for (int q = 0; q < 4; q++) v[q] = epilogue(acc[q][r], alpha, beta, old[q]);
      Vec4<float>::store(cp, v);
    } else {
#pragma unroll
      for (int q = 0; q < 4; q++)
        if (gi + q < m && wg_in_triangle(uplo, gi + q, gj)) {
          const float o = (beta != 0.0f) ? cp[q] : 0.0f;
          cp[q] = epilogue(acc[q][r], alpha, beta, o);
        }
    }
  }
}

// The 16-byte form (lda, ldb multiples of 4, A and B 16-byte aligned): each
// copy moves four elements along the dimension the operand stores
// contiguously, zero-filling past its edge, and shared memory keeps that
// dimension contiguous: op(A) at [p][i] when it is m-contiguous, at [i][p]
// when k-contiguous; op(B) at [j][p] when k-contiguous, at [p][j] when
// n-contiguous. Three copies per thread per k-tile, their source pointers set
// up once. The FMA order per element is the same: p = 0..k-1.
// [row][p] layouts: rows of V_KP floats, the 16-byte chunk at p of row r stored
// at chunk position (p ^ v_swz(r)). A warp reads rows 4t+i for eight (op(A)) or
// four (op(B)) consecutive t; without the swizzle those fall on two bank
// positions, with it on distinct ones.
constexpr int V_KP = S_BK + 4;
__device__ __forceinline__ int v_swz(int r) { return ((r >> 3) & 3) << 2; }
constexpr int V_A = S_BM * V_KP > S_BK * S_LDA ? S_BM * V_KP : S_BK * S_LDA;
constexpr int V_B = S_BN * V_KP > S_BK * S_LDB ? S_BN * V_KP : S_BK * S_LDB;
constexpr int V_STAGE = V_A + V_B;
// A deeper ring than the 4-byte form's: with one CTA per SM (a few hundred
// tiles at most) each k-tile is little work, and the ring must cover the whole
// memory latency of a cold operand.
constexpr int V_STAGES = 12;
constexpr size_t V_SMEM = sizeof(float) * V_STAGES * V_STAGE;

__device__ __forceinline__ void cp_async16(float *dst, const float *src, int bytes) {
  // bytes < 16 zero-fills the rest; 0 reads nothing.
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src), "r"(bytes)
               : "memory");
}

// One 16-byte copy of a tile: smem offset, global source at k-tile 0, its
// advance per k-tile, and how many of its four elements lie inside the matrix
// along the contiguous dimension (0: the row or column is outside).
struct VCopy {
  const float *src;
  int64_t step;
  int dst, valid, pk;  // pk: the copy's first p within a k-tile when p is the contiguous dimension, else -1
  int p;               // its p when p is the strided dimension
};

// Copy q of an operand tile `rows` (the non-k dimension) x S_BK, contiguous
// along the non-k dimension (kcontig = 0: element (r, p) at src[r + p*ld]) or
// along k (kcontig = 1: at src[p + r*ld]).
__device__ __forceinline__ VCopy v_copy(int e, int rows, int kcontig, const float *base, int64_t ld, int64_t r0,
                                        int64_t rlim, int lds_strided) {
  VCopy c;
  if (kcontig) {  // chunks of four p at one row: smem [r][p]
    const int r = e / (S_BK / 4), pc = (e % (S_BK / 4)) * 4;
    const bool in = r0 + r < rlim;
    c.src = in ? base + pc + (r0 + r) * ld : base;
    c.step = in ? S_BK : 0;
    c.dst = r * V_KP + (pc ^ v_swz(r));
    c.valid = in ? 4 : 0;
    c.pk = pc;
    c.p = 0;
  } else {  // chunks of four rows at one p: smem [p][r]
    const int p = e / (rows / 4), rc = (e % (rows / 4)) * 4;
    const int64_t left = rlim - (r0 + rc);
    c.valid = left >= 4 ? 4 : (left > 0 ? (int)left : 0);
    c.src = c.valid ? base + (r0 + rc) + p * ld : base;
    c.step = c.valid ? S_BK * ld : 0;
    c.dst = p * lds_strided + rc;
    c.pk = -1;
    c.p = p;
  }
  return c;
}

// Issues a copy for the k-tile starting at k0, whose source is `src` (the
// copy's source advanced by k0 / S_BK steps): elements at p >= kk are zero-filled.
__device__ __forceinline__ void v_issue(float *tile, const VCopy &c, const float *src, int64_t k0, int64_t kk) {
  int bytes;
  if (c.pk >= 0) {
    const int64_t left = kk - (k0 + c.pk);
    bytes = c.valid == 0 || left <= 0 ? 0 : (left >= 4 ? 16 : (int)left * 4);
  } else {
    bytes = k0 + c.p < kk ? c.valid * 4 : 0;
  }
  cp_async16(tile + c.dst, bytes ? src : c.src, bytes);
}

template <int TA, int TB>
__global__ void __launch_bounds__(S_NT, 2)
gemm_simt_small_vec_kernel(int64_t m, int64_t n, int64_t k, float alpha, const float *__restrict__ A, int64_t lda,
                           const float *__restrict__ B, int64_t ldb, float beta, float *__restrict__ C, int64_t ldc,
                           int uplo) {
  extern __shared__ __align__(16) float sm[];
  const int tid = threadIdx.x, tx = tid % 8, ty = tid / 8;
  const int64_t tiles_m = (m + S_BM - 1) / S_BM;
  const int64_t m0 = (blockIdx.x % tiles_m) * S_BM, n0 = (blockIdx.x / tiles_m) * S_BN;
  if (wg_tile_outside(uplo, m0, S_BM, n0, S_BN)) return;
  const int64_t kk = (alpha == 0.0f) ? 0 : k;
  const int64_t ntiles = (kk + S_BK - 1) / S_BK;

  // op(A): 32 x 16 = 128 chunks (one per thread); op(B): 64 x 16 = 256 (two).
  const VCopy ca = v_copy(tid, S_BM, TA, A, lda, m0, m, S_LDA);
  const VCopy cb0 = v_copy(tid, S_BN, TB ? 0 : 1, B, ldb, n0, n, S_LDB);
  const VCopy cb1 = v_copy(tid + S_NT, S_BN, TB ? 0 : 1, B, ldb, n0, n, S_LDB);
  // The next k-tile to issue: its ring stage, first k and the copies' sources
  // (advanced by one step per tile, so no per-tile index arithmetic).
  int ws = 0;
  int64_t kw = 0;
  const float *pa = ca.src, *pb0 = cb0.src, *pb1 = cb1.src;
  auto issue = [&]() {
    float *as = sm + ws * V_STAGE, *bs = as + V_A;
    v_issue(as, ca, pa, kw, kk);
    v_issue(bs, cb0, pb0, kw, kk);
    v_issue(bs, cb1, pb1, kw, kk);
    pa += ca.step;
    pb0 += cb0.step;
    pb1 += cb1.step;
    kw += S_BK;
    ws = ws + 1 == V_STAGES ? 0 : ws + 1;
  };

  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; i++)
#pragma unroll
    for (int j = 0; j < 4; j++) acc[i][j] = 0.0f;

#pragma unroll
  for (int s = 0; s < V_STAGES - 1; s++) {
    if (s < ntiles) issue();
    cp_async_commit();
  }
  int rs = 0;       // the ring stage of k-tile t
  int64_t rem = kk;  // k values from k-tile t on
  for (int64_t t = 0; t < ntiles; t++, rem -= S_BK) {
    cp_async_wait<V_STAGES - 2>();
    __syncthreads();
    if (t + V_STAGES - 1 < ntiles) issue();
    cp_async_commit();
    const float *as = sm + rs * V_STAGE, *bs = as + V_A;
    rs = rs + 1 == V_STAGES ? 0 : rs + 1;
    // Four p at a time: a[i][q], b[j][q] for rows 4tx+i, columns 4ty+j, p = p0+q.
    auto group = [&](int p0, int np) {
      float a[4][4], b[4][4];
      if (TA) {
#pragma unroll
        for (int i = 0; i < 4; i++) Vec4<float>::load(a[i], as + (4 * tx + i) * V_KP + (p0 ^ v_swz(4 * tx + i)));
      } else {
#pragma unroll
        for (int q = 0; q < 4; q++) {
          float v[4];
          Vec4<float>::load(v, as + (p0 + q) * S_LDA + 4 * tx);
#pragma unroll
          for (int i = 0; i < 4; i++) a[i][q] = v[i];
        }
      }
      if (!TB) {
#pragma unroll
        for (int j = 0; j < 4; j++) Vec4<float>::load(b[j], bs + (4 * ty + j) * V_KP + (p0 ^ v_swz(4 * ty + j)));
      } else {
#pragma unroll
        for (int q = 0; q < 4; q++) {
          float v[4];
          Vec4<float>::load(v, bs + (p0 + q) * S_LDB + 4 * ty);
#pragma unroll
          for (int j = 0; j < 4; j++) b[j][q] = v[j];
        }
      }
#pragma unroll
      for (int q = 0; q < 4; q++)
        if (q < np)
#pragma unroll
          for (int i = 0; i < 4; i++)
#pragma unroll
            for (int j = 0; j < 4; j++) acc[i][j] = __fmaf_rn(a[i][q], b[j][q], acc[i][j]);
    };
    if (rem >= S_BK) {
#pragma unroll
      for (int p0 = 0; p0 < S_BK; p0 += 4) group(p0, 4);
    } else {
      for (int p0 = 0; p0 < (int)rem; p0 += 4) group(p0, (int)rem - p0);
    }
  }
  cp_async_wait<0>();

  const int64_t gi = m0 + 4 * tx;
  if (gi >= m) return;
#pragma unroll
  for (int r = 0; r < 4; r++) {
    const int64_t gj = n0 + 4 * ty + r;
    if (gj >= n) continue;
    float *cp = C + gi + gj * ldc;
    const bool full = gi + 3 < m && (reinterpret_cast<uintptr_t>(cp) % 16 == 0) && wg_in_triangle(uplo, gi, gj) &&
                      wg_in_triangle(uplo, gi + 3, gj);
    if (full) {
      float v[4], old[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      if (beta != 0.0f) Vec4<float>::load(old, cp);
#pragma unroll
      for (int q = 0; q < 4; q++) v[q] = epilogue(acc[q][r], alpha, beta, old[q]);
      Vec4<float>::store(cp, v);
    } else {
#pragma unroll
      for (int q = 0; q < 4; q++)
        if (gi + q < m && wg_in_triangle(uplo, gi + q, gj)) {
          const float o = (beta != 0.0f) ? cp[q] : 0.0f;
          cp[q] = epilogue(acc[q][r], alpha, beta, o);
        }
    }
  }
}

template <int TA, int TB>
cudaError_t launch_small_tt(cudaStream_t s, int64_t m, int64_t n, int64_t k, float alpha, const float *A,
                            int64_t lda, const float *B, int64_t ldb, float beta, float *C, int64_t ldc, int uplo) {
  const int64_t grid = ((m + S_BM - 1) / S_BM) * ((n + S_BN - 1) / S_BN);
  const bool vec = lda % 4 == 0 && ldb % 4 == 0 && reinterpret_cast<uintptr_t>(A) % 16 == 0 &&
                   reinterpret_cast<uintptr_t>(B) % 16 == 0;
  if (vec) {
    auto kern = gemm_simt_small_vec_kernel<TA, TB>;
    cudaError_t e = wg_kernel_smem(kern, V_SMEM, true);
    if (e != cudaSuccess) return e;
    kern<<<(unsigned)grid, S_NT, V_SMEM, s>>>(m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, uplo);
    return cudaGetLastError();
  }
  auto kern = gemm_simt_small_kernel<TA, TB>;
  cudaError_t e = wg_kernel_smem(kern, S_SMEM, true);
  if (e != cudaSuccess) return e;
  kern<<<(unsigned)grid, S_NT, S_SMEM, s>>>(m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, uplo);
  return cudaGetLastError();
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
  // The same shared-memory carveout as the tensor-core kernels it follows, so an
  // SM need not reconfigure between them.
  cudaError_t e = wg_kernel_smem(kern, smem_bytes<T>(), true);
  if (e != cudaSuccess) return e;
  // One CTA per tile; a gated launch (usually a no-op) strides with at most one
  // CTA per SM of a B200, so its closed-gate exit costs little more than the launch.
  int64_t grid = ((m + BM - 1) / BM) * ((n + BN - 1) / BN);
  if (gate && grid > GATED_GRID) grid = GATED_GRID;
  const wg_gate g = gate ? *gate : wg_gate{nullptr, nullptr, 0u, 0u};
  const wg_tile_mask mk = mask ? *mask : wg_tile_mask{nullptr, 1, 1, 0u};
  // A gated launch follows the kernel that sets its gate: it is launched
  // programmatically, so its launch overlaps that kernel's end.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(NT);
  cfg.dynamicSmemBytes = smem_bytes<T>();
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = gate ? 1 : 0;
  const int gated = gate ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, dwords, g, gated, mk, uplo);
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

cudaError_t wg_launch_gemm_simt_small(cudaStream_t s, int transA, int transB, int64_t m, int64_t n, int64_t k,
                                      float alpha, const float *A, int64_t lda, const float *B, int64_t ldb,
                                      float beta, float *C, int64_t ldc, int uplo) {
  if (((m + S_BM - 1) / S_BM) * ((n + S_BN - 1) / S_BN) >= ((int64_t)1 << 31)) return cudaErrorInvalidConfiguration;
  if (transA)
    return transB ? launch_small_tt<1, 1>(s, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, uplo)
                  : launch_small_tt<1, 0>(s, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, uplo);
  return transB ? launch_small_tt<0, 1>(s, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, uplo)
                : launch_small_tt<0, 0>(s, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, uplo);
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
