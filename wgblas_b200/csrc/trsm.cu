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
// FFMA kernels for shallow updates, small shapes and non-finite operands), and
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
// Right-hand sides up to which `auto` takes the flow form.
constexpr int64_t FLOW_AUTO_MAX_RHS = 1024;

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
  // everything else in the tile is zero. All of a thread's loads are issued
  // before its first store (a loop over them one at a time paid a memory
  // latency per element).
  constexpr int PER = LEAF * LEAF / LEAF_RHS;
  float v[PER];
#pragma unroll
  for (int q = 0; q < PER; q++) {
    const int e = threadIdx.x + q * LEAF_RHS;
    const int i = a.l_rs == 1 ? e % LEAF : e / LEAF;  // Lt(i, k) contiguous in i, or in k
    const int k = a.l_rs == 1 ? e / LEAF : e % LEAF;
    const bool below = FORWARD ? i > k : i < k;
    v[q] = (i < nb && k < nb && below) ? a.L[i * a.l_rs + k * a.l_cs] : 0.0f;
  }
#pragma unroll
  for (int q = 0; q < PER; q++) {
    const int e = threadIdx.x + q * LEAF_RHS;
    const int i = a.l_rs == 1 ? e % LEAF : e / LEAF;
    const int k = a.l_rs == 1 ? e / LEAF : e % LEAF;
    Ls[k][i] = v[q];
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

// ---- the flow form: one cooperative launch -----------------------------------
//
// The same substitution-plus-update arithmetic without a launch per block.
// The right-hand sides are cut into chunks of 64; CTA q of a chunk's P owns the
// 64-row blocks p = q, q + P, ... (in solve order) and takes them in turn:
//
//   acc = alpha * Bt[p]                                  (this CTA's block)
//   for each earlier block j:  wait until block j is published,
//                              acc -= Lt[p, j] * Xt[j]   (64 x 64 x 64 FFMA)
//   Xt[p] = substitution on Lt[p, p] over acc; publish block p
//
// Only the owner writes a block, and a block waits only on blocks before it in
// solve order, so with every CTA resident (a cooperative launch) the chain
// always advances. Publishing is a per-(chunk, block) word set to the call's
// epoch after the block's stores (release); a waiter reads it with acquire and
// the block's values bypass L1. Lt[p, j] is loaded before the wait, so only the
// block's own update, its substitution and the publish are on the chain.
// Every element is still alpha*b minus a sum of products times the reciprocal
// of the diagonal, so Infinity and NaN land where substitution puts them.
// Waits are clock-bounded: one that runs out sets WG_DERR_FLOW_WAIT and the CTA
// stops (the blocks it owns stay unsolved; wg_device_check reports it).
constexpr int FLOW_THREADS = 256;
constexpr int FLOW_LD = LEAF + 4;  // shared row stride of the 64 x 64 tiles (16-byte aligned rows)
constexpr long long FLOW_BUDGET = 4000000000LL;  // clock cycles a wait may take (about 2 s)

struct FlowArgs {
  const float *L;  // Lt(r, c) = L[r * l_rs + c * l_cs]
  int64_t l_rs, l_cs;
  float *X;  // Bt(r, o) = X[r * x_rs + o * x_cs]
  int64_t x_rs, x_cs;
  int64_t order, nrhs;
  int nb;      // 64-row blocks
  int chunk0;  // first right-hand-side chunk of this launch
  int P;       // CTAs per chunk
  int unit;
  float alpha;
  unsigned *flags;  // [chunk][nb]
  unsigned epoch;
  unsigned *dwords;
};

// Rows [r0, r0 + len) of block p (solve order).
template <bool FORWARD>
__device__ __forceinline__ void flow_rows(const FlowArgs &a, int p, int64_t &r0, int &len) {
  if (FORWARD) {
    r0 = (int64_t)p * LEAF;
    const int64_t e = r0 + LEAF < a.order ? r0 + LEAF : a.order;
    len = (int)(e - r0);
  } else {
    const int64_t hi = a.order - (int64_t)p * LEAF;
    r0 = hi > LEAF ? hi - LEAF : 0;
    len = (int)(hi - r0);
  }
}

__device__ __forceinline__ unsigned flow_load_acquire(const unsigned *f) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
  return v;
}

__device__ __forceinline__ void flow_store_release(unsigned *f, unsigned v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(f), "r"(v) : "memory");
}

// T[k][i] = Lt(ri + i, rk + k) for i < ni, k < nk (0 elsewhere), in registers
// first (16 per thread) so the loads can be in flight across a wait.
__device__ __forceinline__ void flow_load_l(const FlowArgs &a, int64_t ri, int ni, int64_t rk, int nk, float (&v)[16]) {
#pragma unroll
  for (int t = 0; t < 16; t++) {
    const int e = (int)threadIdx.x + t * FLOW_THREADS;
    int i, k;
    if (a.l_rs == 1) {  // consecutive threads: consecutive rows
      i = e % LEAF;
      k = e / LEAF;
    } else {
      k = e % LEAF;
      i = e / LEAF;
    }
    v[t] = (i < ni && k < nk) ? a.L[(ri + i) * a.l_rs + (rk + k) * a.l_cs] : 0.0f;
  }
}

__device__ __forceinline__ void flow_store_l(const FlowArgs &a, const float (&v)[16], float (*T)[FLOW_LD]) {
#pragma unroll
  for (int t = 0; t < 16; t++) {
    const int e = (int)threadIdx.x + t * FLOW_THREADS;
    const int i = a.l_rs == 1 ? e % LEAF : e / LEAF, k = a.l_rs == 1 ? e / LEAF : e % LEAF;
    T[k][i] = v[t];
  }
}

// T[k][o] = Bt(r + k, o0 + o) for k < n, o < w (0 elsewhere); L1 bypassed.
__device__ __forceinline__ void flow_load_x(const FlowArgs &a, int64_t r, int n, int64_t o0, int w,
                                            float (*T)[FLOW_LD]) {
#pragma unroll
  for (int t = 0; t < 16; t++) {
    const int e = (int)threadIdx.x + t * FLOW_THREADS;
    int k, o;
    if (a.x_rs == 1) {
      k = e % LEAF;
      o = e / LEAF;
    } else {
      o = e % LEAF;
      k = e / LEAF;
    }
    T[k][o] = (k < n && o < w) ? __ldcg(a.X + (r + k) * a.x_rs + (o0 + o) * a.x_cs) : 0.0f;
  }
}

// The diagonal block's referenced side, v[t] = Lt(r0 + i, r0 + k) for
// (i, k) below (FORWARD) or above the diagonal and inside the block, in the
// layout flow_store_l writes.
template <bool FORWARD>
__device__ __forceinline__ void flow_load_diag(const FlowArgs &a, int64_t r0, int len, float (&v)[16]) {
#pragma unroll
  for (int t = 0; t < 16; t++) {
    const int e = (int)threadIdx.x + t * FLOW_THREADS;
    int i, k;
    if (a.l_rs == 1) {
      i = e % LEAF;
      k = e / LEAF;
    } else {
      k = e % LEAF;
      i = e / LEAF;
    }
    const bool side = FORWARD ? i > k : i < k;
    v[t] = (i < len && k < len && side) ? a.L[(r0 + i) * a.l_rs + (r0 + k) * a.l_cs] : 0.0f;
  }
}

template <bool FORWARD>
__global__ void __launch_bounds__(FLOW_THREADS) strsm_flow(FlowArgs a) {
  __shared__ __align__(16) float Ls[LEAF][FLOW_LD];  // update: Ls[k][i] = Lt(p row i, j row k); solve: the diagonal block
  __shared__ __align__(16) float Xs[LEAF][FLOW_LD];  // update: Xs[k][o] = Xt(j row k, o); solve: Xs[o][i]
  __shared__ float rd[LEAF];
  __shared__ int stop;
  const int tid = threadIdx.x, ty = tid / 16, tx = tid % 16;
  const int q = (int)blockIdx.x % a.P;
  const int c = a.chunk0 + (int)blockIdx.x / a.P;
  const int64_t o0 = (int64_t)c * LEAF;
  const int w = (int)(a.nrhs - o0 < LEAF ? a.nrhs - o0 : LEAF);
  unsigned *flags = a.flags + (int64_t)c * a.nb;
  if (tid == 0) stop = 0;
  for (int p = q; p < a.nb; p += a.P) {
    int64_t r0;
    int len;
    flow_rows<FORWARD>(a, p, r0, len);
    // acc = alpha * Bt[p] (this thread's 4 x 4: rows 4ty.., right-hand sides 4tx..)
    __syncthreads();
    flow_load_x(a, r0, len, o0, w, Xs);
    __syncthreads();
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
      for (int j = 0; j < 4; j++) acc[i][j] = a.alpha * Xs[4 * ty + i][4 * tx + j];
    // The diagonal block and its reciprocals, loaded now so that their loads are
    // off the chain.
    float dv[16];
    flow_load_diag<FORWARD>(a, r0, len, dv);
    const float rdv = (tid < len && !a.unit) ? 1.0f / a.L[(r0 + tid) * (a.l_rs + a.l_cs)] : 1.0f;
    for (int jb = 0; jb < p; jb++) {
      int64_t rj;
      int lj;
      flow_rows<FORWARD>(a, jb, rj, lj);
      float lv[16];
      flow_load_l(a, r0, len, rj, lj, lv);  // independent of block jb's values: in flight across the wait
      if (tid == 0) {
        const long long t0 = clock64();
        while (flow_load_acquire(flags + jb) != a.epoch) {
          if (clock64() - t0 > FLOW_BUDGET) {
            atomicOr(a.dwords + WG_DW_ERROR, WG_DERR_FLOW_WAIT);
            stop = 1;
            break;
          }
          __nanosleep(32);
        }
      }
      __syncthreads();  // also: the previous update's reads of Ls / Xs are done
      if (stop) return;  // uniform: every thread read the same word after the barrier
      flow_store_l(a, lv, Ls);
      flow_load_x(a, rj, lj, o0, w, Xs);
      __syncthreads();
#pragma unroll 8
      for (int k = 0; k < LEAF; k++) {
        const float4 l = *reinterpret_cast<const float4 *>(&Ls[k][4 * ty]);
        const float4 x = *reinterpret_cast<const float4 *>(&Xs[k][4 * tx]);
        const float lr[4] = {l.x, l.y, l.z, l.w}, xr[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
          for (int j = 0; j < 4; j++) acc[i][j] = fmaf(-lr[i], xr[j], acc[i][j]);
      }
      __syncthreads();
    }
    // Substitution on the diagonal block (Ls[k][i] = Lt(r0 + i, r0 + k) on the
    // referenced side of the diagonal only, rd[k] its reciprocal diagonal), as in
    // strsm_leaf: one thread per right-hand side.
    flow_store_l(a, dv, Ls);
    if (tid < LEAF) rd[tid] = rdv;
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
      for (int j = 0; j < 4; j++) Xs[4 * tx + j][4 * ty + i] = acc[i][j];  // Xs[o][i]
    __syncthreads();
    if (tid < w) {
      float x[LEAF];
#pragma unroll
      for (int i = 0; i < LEAF; i++) x[i] = Xs[tid][i];
      if (FORWARD) {
#pragma unroll
        for (int k = 0; k < LEAF; k++) {
          if (k < len) {
            const float xk = x[k] * rd[k];
            x[k] = xk;
#pragma unroll
            for (int i = k + 1; i < LEAF; i++) x[i] = fmaf(-Ls[k][i], xk, x[i]);
          }
        }
      } else {
#pragma unroll
        for (int k = LEAF - 1; k >= 0; k--) {
          if (k < len) {
            const float xk = x[k] * rd[k];
            x[k] = xk;
#pragma unroll
            for (int i = 0; i < k; i++) x[i] = fmaf(-Ls[k][i], xk, x[i]);
          }
        }
      }
#pragma unroll
      for (int i = 0; i < LEAF; i++) Xs[tid][i] = x[i];
    }
    __syncthreads();
#pragma unroll
    for (int t = 0; t < 16; t++) {
      const int e = tid + t * FLOW_THREADS;
      int i, o;
      if (a.x_rs == 1) {
        i = e % LEAF;
        o = e / LEAF;
      } else {
        o = e % LEAF;
        i = e / LEAF;
      }
      if (i < len && o < w) a.X[(r0 + i) * a.x_rs + (o0 + o) * a.x_cs] = Xs[o][i];
    }
    __syncthreads();
    if (tid == 0) {
      __threadfence();
      flow_store_release(flags + p, a.epoch);
    }
  }
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

  // C := -op(X) op(Y) + beta C through the sgemm dispatcher: the shallow updates
  // of the lower levels go to the small-tile FFMA kernel (a 64 x 4096 x 64
  // update: 8.8 us against 19.1 on the 128 x 128-tile FFMA kernel, which gives
  // it 32 CTAs), the deeper ones to the tensor cores.
  wg_status gemm(int tX, int tY, int64_t m, int64_t n, int64_t k, const float *X, int64_t ldx, const float *Y,
                 int64_t ldy, float beta, float *C, int64_t ldc) const {
    return wg_gemm_enqueue<float>(d, tX, tY, m, n, k, -1.0f, X, ldx, Y, ldy, beta, C, ldc);
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

  // The whole solve in cooperative launches of strsm_flow (one per group of
  // right-hand-side chunks that fits on the GPU at once).
  wg_status flow(float alpha) const {
    const int64_t nb = (order + LEAF - 1) / LEAF, chunks = (other + LEAF - 1) / LEAF;
    const size_t need = (size_t)nb * (size_t)chunks;
    if (need > d->flow_flags_n) {
      if (d->flow_flags) {
        WG_CUDA(cudaStreamSynchronize(d->stream));  // queued flow launches may still read them
        WG_CUDA(cudaFree(d->flow_flags));
        d->flow_flags = nullptr;
        d->flow_flags_n = 0;
      }
      WG_CUDA(cudaMalloc(&d->flow_flags, need * sizeof(unsigned)));
      WG_CUDA(cudaMemsetAsync(d->flow_flags, 0, need * sizeof(unsigned), d->stream));
      d->flow_flags_n = need;
    }
    if (++d->flow_epoch == 0) ++d->flow_epoch;  // 0 is the allocation's value
    const void *fn = forward ? reinterpret_cast<const void *>(&strsm_flow<true>)
                             : reinterpret_cast<const void *>(&strsm_flow<false>);
    int per_sm = 0;
    WG_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, FLOW_THREADS, 0));
    const int64_t resident = (int64_t)per_sm * d->sm_count;
    if (resident < 1) return wg_fail(WG_ERR_CUDA, "strsm flow kernel cannot be resident");
    // CTAs per chunk: enough to spread the updates, no more than there are blocks.
    int64_t P = resident / chunks;
    if (P > nb) P = nb;
    if (P < 1) P = 1;
    const int64_t group = resident / P;  // chunks per launch
    FlowArgs fa;
    fa.L = A;
    fa.l_rs = l_rs();
    fa.l_cs = l_cs();
    fa.X = B;
    fa.x_rs = b_rs();
    fa.x_cs = b_cs();
    fa.order = order;
    fa.nrhs = other;
    fa.nb = (int)nb;
    fa.P = (int)P;
    fa.unit = unit;
    fa.alpha = alpha;
    fa.flags = d->flow_flags;
    fa.epoch = d->flow_epoch;
    fa.dwords = d->dwords;
    for (int64_t c0 = 0; c0 < chunks; c0 += group) {
      fa.chunk0 = (int)c0;
      const int64_t g = chunks - c0 < group ? chunks - c0 : group;
      void *args[] = {&fa};
      wg_launch_scope scope(d, "strsm_flow");
      WG_CUDA(cudaLaunchCooperativeKernel(fn, dim3((unsigned)(g * P)), dim3(FLOW_THREADS), args, 0, d->stream));
    }
    return WG_OK;
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

// AUTO: the flow form when the solve has more than one block and few
// right-hand sides, where the recursive form's many small launches dominate.
bool use_flow(const wg_device *d, int64_t order, int64_t other) {
  if (d->strsm_path == WG_STRSM_FLOW) return true;
  if (d->strsm_path == WG_STRSM_RECURSIVE) return false;
  return order > LEAF && other <= FLOW_AUTO_MAX_RHS;
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
    if (use_flow(d, t.order, t.other)) {
      st = t.flow(alpha);
    } else if (t.order > LEAF && wg_tf32x3_supported(d, t.order, t.other, t.order)) {
      // Size the GEMM scratch for the largest update up front: growing it
      // later would wait for the queued solve.
      void *ws = nullptr;
      st = wg_workspace(d, wg_tf32x3_workspace_bytes_sk(d, t.order, t.other, t.order), &ws);
      if (st == WG_OK) st = t.solve(0, t.order, alpha);
    } else {
      st = t.solve(0, t.order, alpha);
    }
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
