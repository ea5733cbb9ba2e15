// strsm: B := alpha * op(A)^-1 * B (side left) or alpha * B * op(A)^-1 (side
// right), A triangular, in the column-major BLAS frame. The reference routine is
// src/strsm/strsm.mjs:160-583; the host layer maps its row-major calls onto
// this frame.
//
// Solve frame. Both sides are written as one lower-or-upper system
// Lt * Xt = Bt over the "blocked" axis: for side left Lt = op(A) and Bt = B (the
// right-hand sides are B's columns); for side right Lt = op(A)^T and Bt = B^T
// (X * op(A) = B is op(A)^T * X^T = B^T, the right-hand sides are B's rows).
// The solve runs forward when Lt is lower and backward when it is upper.
//
// Recursive blocked solve. The order-`order` triangle is halved (at multiples
// of 64) until a diagonal block has at most 64 rows:
//
//   solve(first half, alpha)
//   Bt[second] := alpha * Bt[second] - Lt[second, first] * Xt[first]   (one GEMM)
//   solve(second half, 1)
//
// so the m*n*order multiply-adds run almost entirely in a few large GEMMs
// (the 3xTF32 tensor-core path for the deep updates of the upper levels, the
// FFMA kernel for shallow updates, small shapes and non-finite operands), and
// the diagonal blocks in `strsm_leaf`. The reference instead
// walks 64-row blocks one at a time with a k=64 update GEMM after each
// (strsm.mjs:399-432) and, above eight blocks, applies explicit block inverses
// (strsv_invert_block.wgsl). Substitution plus GEMM keeps stdlib's IEEE
// placement of Infinity and NaN for every input: every element is
// alpha*b minus a sum of products and a division by the diagonal, and the
// class of such a sum (finite, +-Infinity, NaN) does not depend on the order of
// its terms.
//
// The leaf kernel is latency-bound (a 64-step dependency chain per right-hand
// side); it keeps one right-hand side's 64 unknowns in registers per thread,
// updates them column by column (axpy form: after x_k is final, every later
// unknown subtracts L(i,k) * x_k, 63 independent FMAs per step), and reads the
// block of Lt from shared memory as broadcasts.
#include "internal.h"

namespace {

constexpr int LEAF = 64;      // rows of a diagonal block
constexpr int LEAF_RHS = 64;  // right-hand sides per CTA, one per thread
constexpr int LS = LEAF + 4;  // shared row stride: keeps 16-byte alignment of each column
// Updates at most this deep (the lower levels of the recursion) run on the FFMA
// kernel: the tensor-core path costs a split pass plus a fixed time per call in
// its MMA kernel (68 us for a 512^3 product, measured with per-kernel events)
// that a k <= 256 update does not amortise.
constexpr int64_t SIMT_MAX_K = 256;

struct LeafArgs {
  const float *L;  // Lt(0, 0) of the diagonal block
  int64_t l_rs, l_cs;
  float *X;  // Bt(0, 0) of the block's rows
  int64_t x_rs, x_cs;
  int64_t nrhs;
  int nb;  // rows of this block, 1..LEAF
  int unit;
  float alpha;
};

// FORWARD: Lt lower, unknowns in increasing order; else Lt upper, decreasing.
template <bool FORWARD>
__global__ void __launch_bounds__(LEAF_RHS) strsm_leaf(LeafArgs a) {
  // Ls[k][i] = Lt(i, k): column k of the block contiguous, read as broadcasts.
  __shared__ __align__(16) float Ls[LEAF][LS];
  __shared__ float rd[LEAF];
  const int nb = a.nb;
  // Only the referenced triangle is read (the other one may hold anything);
  // everything else in the tile is zero.
  for (int e = threadIdx.x; e < LEAF * LEAF; e += blockDim.x) {
    int i, k;
    if (a.l_rs == 1) {  // Lt(i, k) contiguous in i
      i = e % LEAF;
      k = e / LEAF;
    } else {
      k = e % LEAF;
      i = e / LEAF;
    }
    const bool below = FORWARD ? i > k : i < k;
    float v = 0.0f;
    if (i < nb && k < nb && below) v = a.L[i * a.l_rs + k * a.l_cs];
    Ls[k][i] = v;
  }
  for (int k = threadIdx.x; k < LEAF; k += blockDim.x)
    rd[k] = (k < nb && !a.unit) ? 1.0f / a.L[k * (a.l_rs + a.l_cs)] : 1.0f;
  __syncthreads();

  const int64_t o = (int64_t)blockIdx.x * LEAF_RHS + threadIdx.x;
  if (o >= a.nrhs) return;
  float *xp = a.X + o * a.x_cs;
  float x[LEAF];
#pragma unroll
  for (int i = 0; i < LEAF; i++) x[i] = i < nb ? a.alpha * xp[i * a.x_rs] : 0.0f;
  if (FORWARD) {
#pragma unroll
    for (int k = 0; k < LEAF; k++) {
      if (k < nb) {
        const float xk = x[k] * rd[k];
        x[k] = xk;
#pragma unroll
        for (int i = k + 1; i < LEAF; i++) x[i] = fmaf(-Ls[k][i], xk, x[i]);
      }
    }
  } else {
#pragma unroll
    for (int k = LEAF - 1; k >= 0; k--) {
      if (k < nb) {
        const float xk = x[k] * rd[k];
        x[k] = xk;
#pragma unroll
        for (int i = 0; i < k; i++) x[i] = fmaf(-Ls[k][i], xk, x[i]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < LEAF; i++)
    if (i < nb) xp[i * a.x_rs] = x[i];
}

// The problem in the solve frame, with every pointer already at its offset.
struct Trsm {
  wg_device *d;
  int left, trans, forward, unit;
  int64_t order, other;  // order of the triangle, number of right-hand sides
  const float *A;
  int64_t lda;
  float *B;
  int64_t ldb;

  // Lt(r, c) = L[r * rs + c * cs]
  int64_t l_rs() const { return left ? (trans ? lda : 1) : (trans ? 1 : lda); }
  int64_t l_cs() const { return left ? (trans ? 1 : lda) : (trans ? lda : 1); }
  // Bt(r, o) = B[r * rs + o * cs]
  int64_t b_rs() const { return left ? 1 : ldb; }
  int64_t b_cs() const { return left ? ldb : 1; }

  wg_status leaf(int64_t r0, int64_t nb, float alpha) const {
    LeafArgs a;
    a.L = A + r0 * (l_rs() + l_cs());
    a.l_rs = l_rs();
    a.l_cs = l_cs();
    a.X = B + r0 * b_rs();
    a.x_rs = b_rs();
    a.x_cs = b_cs();
    a.nrhs = other;
    a.nb = (int)nb;
    a.unit = unit;
    a.alpha = alpha;
    wg_launch_scope scope(d, "strsm_leaf");
    const unsigned grid = (unsigned)((other + LEAF_RHS - 1) / LEAF_RHS);
    if (forward)
      strsm_leaf<true><<<grid, LEAF_RHS, 0, d->stream>>>(a);
    else
      strsm_leaf<false><<<grid, LEAF_RHS, 0, d->stream>>>(a);
    WG_CUDA(cudaGetLastError());
    return WG_OK;
  }

  // C := -op(X) op(Y) + beta C, on the FFMA kernel when k is shallow.
  wg_status gemm(int tX, int tY, int64_t m, int64_t n, int64_t k, const float *X, int64_t ldx, const float *Y,
                 int64_t ldy, float beta, float *C, int64_t ldc) const {
    if (k > SIMT_MAX_K || d->sgemm_path == WG_SGEMM_TF32X3)
      return wg_gemm_enqueue<float>(d, tX, tY, m, n, k, -1.0f, X, ldx, Y, ldy, beta, C, ldc);
    if (m == 0 || n == 0) return WG_OK;
    d->stats.calls++;
    d->stats.simt_launches++;
    wg_launch_scope scope(d, "sgemm_simt");
    WG_CUDA(wg_launch_gemm_simt<float>(d->stream, tX, tY, m, n, k, -1.0f, X, ldx, Y, ldy, beta, C, ldc, d->dwords,
                                       nullptr));
    return WG_OK;
  }

  // Bt[R] := beta * Bt[R] - Lt[R, J] * Xt[J], R = [r0, r0 + nr), J = [j0, j0 + nj).
  wg_status update(int64_t r0, int64_t nr, int64_t j0, int64_t nj, float beta) const {
    if (left) {
      // B[R, :] -= op(A)[R, J] * B[J, :]; op(A)[R, J] is A[R, J] or A[J, R]^T.
      const float *ap = trans ? A + j0 + r0 * lda : A + r0 + j0 * lda;
      return gemm(trans, 0, nr, other, nj, ap, lda, B + j0, ldb, beta, B + r0, ldb);
    }
    // B[:, R] -= B[:, J] * op(A)[J, R]; op(A)[J, R] is A[J, R] or A[R, J]^T.
    const float *ap = trans ? A + r0 + j0 * lda : A + j0 + r0 * lda;
    return gemm(0, trans, other, nr, nj, B + j0 * ldb, ldb, ap, lda, beta, B + r0 * ldb, ldb);
  }

  wg_status solve(int64_t lo, int64_t hi, float alpha) const {
    const int64_t len = hi - lo;
    if (len <= LEAF) return leaf(lo, len, alpha);
    const int64_t h = ((len / 2 + LEAF - 1) / LEAF) * LEAF;  // first part, a multiple of LEAF
    const int64_t f0 = forward ? lo : hi - h, f1 = f0 + h;    // solved first
    const int64_t s0 = forward ? f1 : lo, s1 = forward ? hi : f0;
    wg_status st = solve(f0, f1, alpha);
    if (st == WG_OK) st = update(s0, s1 - s0, f0, h, alpha);
    if (st == WG_OK) st = solve(s0, s1, 1.0f);
    return st;
  }
};

wg_status check_args(wg_device *d, int side, int uplo, int transA, int diag, int64_t m, int64_t n, int64_t lda,
                     int64_t ldb) {
  if (!d) return wg_fail(WG_ERR_INVALID_ARGUMENT, "device is NULL");
  if (side != WG_SIDE_LEFT && side != WG_SIDE_RIGHT)
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "side must be 'left' or 'right'.");
  if (uplo != WG_UPLO_LOWER && uplo != WG_UPLO_UPPER)
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "uplo must be 'lower' or 'upper'.");
  if (transA != 0 && transA != 1)
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "transA must be 0 (no-transpose) or 1 (transpose)");
  if (diag != WG_DIAG_NON_UNIT && diag != WG_DIAG_UNIT)
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "diag must be 'unit' or 'non-unit'.");
  if (m < 0 || n < 0) return wg_fail(WG_ERR_INVALID_ARGUMENT, "m and n must be non-negative.");
  if (lda <= 0 || ldb <= 0) return wg_fail(WG_ERR_INVALID_ARGUMENT, "lda and ldb must be positive.");
  const int64_t lim = (int64_t)1 << 31, ld_lim = (int64_t)1 << 40;
  if (m >= lim || n >= lim || lda >= ld_lim || ldb >= ld_lim)
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "dimensions must be below 2^31 and leading dimensions below 2^40");
  if (m == 0 || n == 0) return WG_OK;
  if (lda < (side == WG_SIDE_LEFT ? m : n))
    return wg_fail(WG_ERR_INVALID_ARGUMENT, side == WG_SIDE_LEFT ? "lda must be >= m." : "lda must be >= n.");
  if (ldb < m) return wg_fail(WG_ERR_INVALID_ARGUMENT, "ldb must be >= rows of B as stored.");
  if (d->cc_major != 10)
    return wg_fail(WG_ERR_NOT_SUPPORTED, "device %d (%s) is not a Blackwell sm_100 device", d->ordinal, d->name);
  return WG_OK;
}

bool fits(const wg_buffer *b, int64_t off, int64_t rows, int64_t cols, int64_t ld) {
  if (!b || off < 0) return false;
  const __int128 last = (__int128)off + (__int128)(cols - 1) * ld + rows;
  return last * (__int128)sizeof(float) <= (__int128)b->bytes;
}

wg_status strsm_enqueue(wg_device *d, int side, int uplo, int transA, int diag, int64_t m, int64_t n, float alpha,
                        const float *A, int64_t lda, float *B, int64_t ldb, float *gpu_ms) {
  const bool timing = gpu_ms && (d->flags & WG_DEVICE_TIMING);
  if (timing) WG_CUDA(cudaEventRecord(d->ev_start, d->stream));
  wg_status st = WG_OK;
  if (alpha == 0.0f) {
    // BLAS: alpha = 0 makes B a literal zero without reading A or B
    // (strsm.mjs:373-378).
    wg_launch_scope scope(d, "scale");
    WG_CUDA(wg_launch_scale<float>(d->stream, m, n, 0.0f, 0.0f, B, ldb));
  } else {
    const int left = side == WG_SIDE_LEFT;
    const int op_lower = (transA == 0) == (uplo == WG_UPLO_LOWER);
    Trsm t{d, left, transA, left ? op_lower : !op_lower, diag == WG_DIAG_UNIT, left ? m : n, left ? n : m,
           A, lda, B, ldb};
    if (t.order > LEAF && wg_tf32x3_supported(d, t.order, t.other, t.order)) {
      // Size the GEMM scratch for the largest update up front: growing it
      // later would wait for the queued solve.
      void *ws = nullptr;
      st = wg_workspace(d, wg_tf32x3_workspace_bytes_sk(d, t.order, t.other, t.order), &ws);
    }
    if (st == WG_OK) st = t.solve(0, t.order, alpha);
  }
  if (st != WG_OK) return st;
  if (timing) {
    WG_CUDA(cudaEventRecord(d->ev_stop, d->stream));
    WG_CUDA(cudaEventSynchronize(d->ev_stop));
    WG_CUDA(cudaEventElapsedTime(gpu_ms, d->ev_start, d->ev_stop));
  }
  return WG_OK;
}

}  // namespace

extern "C" wg_status wg_strsm(wg_device *d, int side, int uplo, int transA, int diag, int64_t m, int64_t n,
                              float alpha, const wg_buffer *A, int64_t offA, int64_t lda, wg_buffer *B, int64_t offB,
                              int64_t ldb, float *gpu_ms) {
  if (gpu_ms) *gpu_ms = 0.0f;
  wg_status st = check_args(d, side, uplo, transA, diag, m, n, lda, ldb);
  if (st != WG_OK || m == 0 || n == 0) return st;
  const int64_t order = side == WG_SIDE_LEFT ? m : n;
  if (!B || !fits(B, offB, m, n, ldb))
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "B does not have enough elements for the given dimensions and ldb.");
  if (alpha != 0.0f && (!A || !fits(A, offA, order, order, lda)))
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "A does not have enough elements for the given dimensions and lda.");
  if (B->dev->ordinal != d->ordinal || (alpha != 0.0f && A->dev->ordinal != d->ordinal))
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "a buffer belongs to another device");
  wg_device_guard guard(d->ordinal);
  return strsm_enqueue(d, side, uplo, transA, diag, m, n, alpha,
                       alpha != 0.0f ? static_cast<const float *>(A->ptr) + offA : nullptr, lda,
                       static_cast<float *>(B->ptr) + offB, ldb, gpu_ms);
}

extern "C" wg_status wg_strsm_dev(wg_device *d, int side, int uplo, int transA, int diag, int64_t m, int64_t n,
                                  float alpha, const float *A, int64_t lda, float *B, int64_t ldb) {
  wg_status st = check_args(d, side, uplo, transA, diag, m, n, lda, ldb);
  if (st != WG_OK || m == 0 || n == 0) return st;
  if (!B || (alpha != 0.0f && !A)) return wg_fail(WG_ERR_INVALID_ARGUMENT, "operand pointer is NULL");
  wg_device_guard guard(d->ordinal);
  return strsm_enqueue(d, side, uplo, transA, diag, m, n, alpha, A, lda, B, ldb, nullptr);
}
