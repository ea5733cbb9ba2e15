// sgemv / dgemv: y := alpha * op(A) * x + beta * y in the column-major BLAS
// frame (A is m x n, lda >= m). The reference routines are src/sgemv/sgemv.mjs
// and src/dgemv/dgemv.mjs with sgemv_n.wgsl / sgemv_t.wgsl (and the
// double-double twins); their row-major kernel frame is this frame transposed,
// so the reference's "no-transpose" kernel is trans = 1 here and its
// "transpose" kernel trans = 0.
//
// Both shapes are HBM-bound (each element of A is read once, 2 FLOPs per
// element), so the kernels are built for coalescing and loads in flight:
//
// * trans = 1, y_j = sum_i A(i, j) x_i: column j is contiguous. A CTA of 256
//   threads walks one column at a time (grid-stride over columns), each thread
//   with four independent accumulators over rows i, i+256, i+512, i+768, then a
//   warp-shuffle and shared-memory reduction in a fixed order. When there are
//   too few columns to fill the GPU the rows are cut into chunks (blockIdx.y)
//   whose partial sums a second kernel adds in chunk order.
// * trans = 0, y_i = sum_j A(i, j) x_j: one thread per row i (consecutive
//   threads read consecutive addresses of each column), four independent
//   accumulators over columns, and the columns cut into chunks (blockIdx.y)
//   so that enough threads are in flight, summed in chunk order by the same
//   second kernel. A column whose x entry is +-0 adds exactly 0, as reference
//   BLAS skips it (sgemv_t.wgsl:37-46): Infinity or NaN in such a column never
//   meets that zero.
//
// Epilogue (sgemv_n.wgsl:67-73): acc = alpha * sum; y = acc + beta * y when
// beta != 0, else acc (y not read). alpha = 0 scales y by beta without reading
// A or x (y = 0 when beta = 0); alpha = 0 with beta = 1 returns at once.
// The partial sums of several chunks live in the device workspace.
#include "internal.h"

namespace {

constexpr int GEMV_THREADS = 256;

__device__ __forceinline__ float fma_v(float a, float b, float c) { return fmaf(a, b, c); }
__device__ __forceinline__ double fma_v(double a, double b, double c) { return fma(a, b, c); }

template <typename T>
__device__ __forceinline__ T finish(T sum, T alpha, T beta, const T *yp) {
  const T acc = alpha * sum;
  return beta != T(0) ? fma_v(beta, *yp, acc) : acc;
}

// trans = 1. Rows [c * rows, min(m, (c + 1) * rows)) of chunk c = blockIdx.y.
template <typename T>
__global__ void __launch_bounds__(GEMV_THREADS)
    gemv_dot_kernel(int64_t m, int64_t n, const T *__restrict__ A, int64_t lda, const T *__restrict__ x,
                    int64_t incx, int64_t rows, int chunks, T alpha, T beta, T *__restrict__ y, int64_t incy,
                    T *__restrict__ partial) {
  wg_pdl_wait();     // launched programmatically: the kernel before this one has finished
  wg_pdl_trigger();  // and the next gemv launch may be scheduled
  __shared__ T red[GEMV_THREADS / 32];
  const int64_t i0 = (int64_t)blockIdx.y * rows;
  const int64_t i1 = i0 + rows < m ? i0 + rows : m;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int64_t j = blockIdx.x; j < n; j += gridDim.x) {  // uniform per CTA
    const T *col = A + j * lda;
    T a0 = T(0), a1 = T(0), a2 = T(0), a3 = T(0);
    int64_t i = i0 + threadIdx.x;
    for (; i + 3 * GEMV_THREADS < i1; i += 4 * GEMV_THREADS) {
      a0 = fma_v(col[i], x[i * incx], a0);
      a1 = fma_v(col[i + GEMV_THREADS], x[(i + GEMV_THREADS) * incx], a1);
      a2 = fma_v(col[i + 2 * GEMV_THREADS], x[(i + 2 * GEMV_THREADS) * incx], a2);
      a3 = fma_v(col[i + 3 * GEMV_THREADS], x[(i + 3 * GEMV_THREADS) * incx], a3);
    }
    for (; i < i1; i += GEMV_THREADS) a0 = fma_v(col[i], x[i * incx], a0);
    T s = (a0 + a1) + (a2 + a3);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) red[warp] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
      T t = red[0];
#pragma unroll
      for (int w = 1; w < GEMV_THREADS / 32; w++) t += red[w];
      if (chunks == 1)
        y[j * incy] = finish(t, alpha, beta, y + j * incy);
      else
        partial[(int64_t)blockIdx.y * n + j] = t;
    }
    __syncthreads();  // red[] is reused by the next column
  }
}

// 16-byte vectors of T: four floats or two doubles.
template <typename T>
struct V16;
template <>
struct V16<float> {
  using type = float4;
  static constexpr int N = 4;
  __device__ __forceinline__ static float dot(float4 a, float4 b, float acc) {
    return fmaf(a.w, b.w, fmaf(a.z, b.z, fmaf(a.y, b.y, fmaf(a.x, b.x, acc))));
  }
};
template <>
struct V16<double> {
  using type = double2;
  static constexpr int N = 2;
  __device__ __forceinline__ static double dot(double2 a, double2 b, double acc) {
    return fma(a.y, b.y, fma(a.x, b.x, acc));
  }
};

// trans = 1 with 16-byte aligned columns and unit-stride x: one warp per column
// j = blockIdx.x * 8 + warp (no block barrier), each lane reading eight 16-byte
// vectors per step, software-pipelined (the next step's loads are issued before
// this step's FMAs), so that every SM keeps tens of KB of loads in flight.
// Rows [c * rows, ...) of chunk c = blockIdx.y, rows a multiple of the vector
// width.
template <typename T>
__global__ void __launch_bounds__(GEMV_THREADS, 2)
    gemv_dot_vec_kernel(int64_t m, int64_t n, const T *__restrict__ A, int64_t lda, const T *__restrict__ x,
                        int64_t rows, int chunks, T alpha, T beta, T *__restrict__ y, int64_t incy,
                        T *__restrict__ partial) {
  wg_pdl_wait();     // launched programmatically: the kernel before this one has finished
  wg_pdl_trigger();  // and the next gemv launch may be scheduled
  using V = typename V16<T>::type;
  constexpr int W = V16<T>::N, U = 8;
  const int lane = threadIdx.x & 31;
  const int64_t j = (int64_t)blockIdx.x * (GEMV_THREADS / 32) + (threadIdx.x >> 5);  // one column per warp
  if (j >= n) return;  // no barriers below
  const int64_t i0 = (int64_t)blockIdx.y * rows;
  const int64_t i1 = i0 + rows < m ? i0 + rows : m;
  const int64_t v1 = i1 / W;  // whole vectors; the rest (< W rows) by lane 0
  const V *xv = reinterpret_cast<const V *>(x);
  const T *col = A + j * lda;
  const V *cv = reinterpret_cast<const V *>(col);
  T acc[4] = {T(0), T(0), T(0), T(0)};
  int64_t v = i0 / W + lane;
  if (v + 32 * (U - 1) < v1) {
    V c[U];
#pragma unroll
    for (int u = 0; u < U; u++) c[u] = __ldcs(cv + v + 32 * u);
    for (;;) {
      const int64_t nv = v + 32 * U;
      const bool more = nv + 32 * (U - 1) < v1;
      V d[U];
      if (more) {
#pragma unroll
        for (int u = 0; u < U; u++) d[u] = __ldcs(cv + nv + 32 * u);
      }
#pragma unroll
      for (int u = 0; u < U; u++) acc[u & 3] = V16<T>::dot(c[u], __ldg(xv + v + 32 * u), acc[u & 3]);
      v = nv;
      if (!more) break;
#pragma unroll
      for (int u = 0; u < U; u++) c[u] = d[u];
    }
  }
  for (; v < v1; v += 32) acc[0] = V16<T>::dot(__ldcs(cv + v), __ldg(xv + v), acc[0]);
  if (lane == 0)
    for (int64_t i = v1 * W; i < i1; i++) acc[0] = fma_v(col[i], x[i], acc[0]);
  T s = (acc[0] + acc[1]) + (acc[2] + acc[3]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) {
    if (chunks == 1)
      y[j * incy] = finish(s, alpha, beta, y + j * incy);
    else
      partial[(int64_t)blockIdx.y * n + j] = s;
  }
}

// trans = 0 with 16-byte aligned columns and too few rows for gemv_rows_kernel:
// each thread owns W consecutive rows (one 16-byte vector of every column) and
// walks four columns per step. A column whose x entry is +-0 adds nothing (its
// loads are issued regardless, so they never wait on x).
// Rows of the tail (m not a multiple of W) go to gemv_axpy_kernel.
template <typename T>
__global__ void __launch_bounds__(GEMV_THREADS)
    gemv_axpy_vec_kernel(int64_t mv, int64_t n, const T *__restrict__ A, int64_t lda, const T *__restrict__ x,
                         int64_t incx, int64_t cols, int chunks, int64_t ylen, T alpha, T beta, T *__restrict__ y,
                         int64_t incy, T *__restrict__ partial) {
  wg_pdl_wait();     // launched programmatically: the kernel before this one has finished
  wg_pdl_trigger();  // and the next gemv launch may be scheduled
  using V = typename V16<T>::type;
  constexpr int W = V16<T>::N;
  const int64_t t = (int64_t)blockIdx.x * GEMV_THREADS + threadIdx.x;  // vector row index
  if (t >= mv) return;  // no barriers below
  const int64_t j0 = (int64_t)blockIdx.y * cols;
  const int64_t j1 = j0 + cols < n ? j0 + cols : n;
  T acc[W];
#pragma unroll
  for (int q = 0; q < W; q++) acc[q] = T(0);
  const V *a = reinterpret_cast<const V *>(A) + t;
  const int64_t ldv = lda / W;
  int64_t j = j0;
  for (; j + 3 < j1; j += 4) {
    const T x0 = x[j * incx], x1 = x[(j + 1) * incx], x2 = x[(j + 2) * incx], x3 = x[(j + 3) * incx];
    const V c0 = __ldcs(a + j * ldv), c1 = __ldcs(a + (j + 1) * ldv);
    const V c2 = __ldcs(a + (j + 2) * ldv), c3 = __ldcs(a + (j + 3) * ldv);
    const T *e0 = reinterpret_cast<const T *>(&c0), *e1 = reinterpret_cast<const T *>(&c1);
    const T *e2 = reinterpret_cast<const T *>(&c2), *e3 = reinterpret_cast<const T *>(&c3);
#pragma unroll
    for (int q = 0; q < W; q++) {
      if (x0 != T(0)) acc[q] = fma_v(e0[q], x0, acc[q]);
      if (x1 != T(0)) acc[q] = fma_v(e1[q], x1, acc[q]);
      if (x2 != T(0)) acc[q] = fma_v(e2[q], x2, acc[q]);
      if (x3 != T(0)) acc[q] = fma_v(e3[q], x3, acc[q]);
    }
  }
  for (; j < j1; j++) {
    const T xj = x[j * incx];
    if (xj != T(0)) {
      const V c = a[j * ldv];
      const T *e = reinterpret_cast<const T *>(&c);
#pragma unroll
      for (int q = 0; q < W; q++) acc[q] = fma_v(e[q], xj, acc[q]);
    }
  }
#pragma unroll
  for (int q = 0; q < W; q++) {
    const int64_t i = t * W + q;
    if (chunks == 1)
      y[i * incy] = finish(acc[q], alpha, beta, y + i * incy);
    else
      partial[(int64_t)blockIdx.y * ylen + i] = acc[q];
  }
}

// trans = 0 with 16-byte aligned columns and rows enough to fill the GPU: one
// CTA of 512 threads per block of R = W * L consecutive rows and every column,
// so no partial sums leave the CTA. Thread (g, l) = (threadIdx.x / L,
// threadIdx.x % L) owns rows [r0 + l * W, +W) and walks columns g, g + G,
// g + 2G, ... (G = 512 / L column groups) eight at a time, software-pipelined:
// the eight 16-byte loads of the next step are issued before the current step's
// FMAs, so every thread keeps 8 to 16 loads in flight throughout. Each warp
// request reads 32 / L column segments of L * 16 bytes. The G partial vectors
// are then added in shared memory in a fixed order: slice s of W consecutive
// groups by S = 512 / R threads per row, then the S slice sums in order.
// A is loaded whatever x holds; a column whose x entry is +-0 adds nothing.
// UNIT_X (incx = 1) keeps the x offsets compile-time constants: the general
// stride's multiply measured 10% slower at 4096 x 4096.
// The vector that holds row m - 1 may run past the last column's storage, so the
// thread that owns it reads its rows one element at a time.
constexpr int ROWS_THREADS = 512;

template <typename T, int L, bool UNIT_X>
__global__ void __launch_bounds__(ROWS_THREADS)
    gemv_rows_kernel(int64_t m, int64_t n, const T *__restrict__ A, int64_t lda, const T *__restrict__ x,
                     int64_t incx, T alpha, T beta, T *__restrict__ y, int64_t incy) {
  wg_pdl_wait();     // launched programmatically: the kernel before this one has finished
  wg_pdl_trigger();  // and the next gemv launch may be scheduled
  using V = typename V16<T>::type;
  constexpr int W = V16<T>::N, G = ROWS_THREADS / L, R = W * L, S = ROWS_THREADS / R, U = 8;
  static_assert(G % S == 0, "slices must split the column groups evenly");
  __shared__ __align__(16) T part[G * R];
  __shared__ T slice[S * R];
  const int l = threadIdx.x % L, g = threadIdx.x / L;
  const int64_t r0 = (int64_t)blockIdx.x * R;
  const int64_t i = r0 + (int64_t)l * W;
  const int64_t valid = m - i;  // rows of this thread's vector inside A
  T acc[W];
#pragma unroll
  for (int q = 0; q < W; q++) acc[q] = T(0);
  int64_t j = g;
  if (valid >= W) {
    const T *a = A + i;
    if (j + (U - 1) * G < n) {
      V c[U];
#pragma unroll
      for (int u = 0; u < U; u++) c[u] = __ldcs(reinterpret_cast<const V *>(a + (j + u * G) * lda));
      for (;;) {
        const int64_t nj = j + U * G;
        const bool more = nj + (U - 1) * G < n;
        V d[U];
        if (more) {
#pragma unroll
          for (int u = 0; u < U; u++) d[u] = __ldcs(reinterpret_cast<const V *>(a + (nj + u * G) * lda));
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
          const T xj = UNIT_X ? x[j + u * G] : x[(j + u * G) * incx];
          const T *e = reinterpret_cast<const T *>(&c[u]);
#pragma unroll
          for (int q = 0; q < W; q++) acc[q] = xj != T(0) ? fma_v(e[q], xj, acc[q]) : acc[q];
        }
        j = nj;
        if (!more) break;
#pragma unroll
        for (int u = 0; u < U; u++) c[u] = d[u];
      }
    }
    for (; j < n; j += G) {
      const V c = __ldcs(reinterpret_cast<const V *>(a + j * lda));
      const T xj = x[j * incx];
      const T *e = reinterpret_cast<const T *>(&c);
      if (xj != T(0)) {
#pragma unroll
        for (int q = 0; q < W; q++) acc[q] = fma_v(e[q], xj, acc[q]);
      }
    }
  } else if (valid > 0) {
    for (; j < n; j += G) {
      const T xj = x[j * incx];
      if (xj != T(0)) {
#pragma unroll
        for (int q = 0; q < W; q++)
          if (q < valid) acc[q] = fma_v(A[i + q + j * lda], xj, acc[q]);
      }
    }
  }
  V out;
  T *o = reinterpret_cast<T *>(&out);
#pragma unroll
  for (int q = 0; q < W; q++) o[q] = acc[q];
  reinterpret_cast<V *>(part)[threadIdx.x] = out;  // part[g * R + l * W + q]
  __syncthreads();
  {
    const int r = threadIdx.x % R, sl = threadIdx.x / R;
    T s = T(0);
#pragma unroll
    for (int k = 0; k < G / S; k++) s += part[(sl * (G / S) + k) * R + r];
    slice[sl * R + r] = s;
  }
  __syncthreads();
  if (threadIdx.x < R) {
    const int64_t row = r0 + threadIdx.x;
    if (row < m) {
      T s = T(0);
#pragma unroll
      for (int k = 0; k < S; k++) s += slice[k * R + threadIdx.x];
      y[row * incy] = finish(s, alpha, beta, y + row * incy);
    }
  }
}

// trans = 0. Columns [c * cols, min(n, (c + 1) * cols)) of chunk c = blockIdx.y.
template <typename T>
__global__ void __launch_bounds__(GEMV_THREADS)
    gemv_axpy_kernel(int64_t i_begin, int64_t m, int64_t n, const T *__restrict__ A, int64_t lda,
                     const T *__restrict__ x, int64_t incx, int64_t cols, int chunks, T alpha, T beta,
                     T *__restrict__ y, int64_t incy, T *__restrict__ partial) {
  wg_pdl_wait();     // launched programmatically: the kernel before this one has finished
  wg_pdl_trigger();  // and the next gemv launch may be scheduled
  const int64_t i = i_begin + (int64_t)blockIdx.x * GEMV_THREADS + threadIdx.x;
  if (i >= m) return;  // no barriers below
  const int64_t j0 = (int64_t)blockIdx.y * cols;
  const int64_t j1 = j0 + cols < n ? j0 + cols : n;
  const T *a = A + i;
  T a0 = T(0), a1 = T(0), a2 = T(0), a3 = T(0);
  int64_t j = j0;
  for (; j + 3 < j1; j += 4) {
    const T x0 = x[j * incx], x1 = x[(j + 1) * incx], x2 = x[(j + 2) * incx], x3 = x[(j + 3) * incx];
    const T v0 = a[j * lda], v1 = a[(j + 1) * lda], v2 = a[(j + 2) * lda], v3 = a[(j + 3) * lda];
    a0 = fma_v(x0 == T(0) ? T(0) : v0, x0, a0);
    a1 = fma_v(x1 == T(0) ? T(0) : v1, x1, a1);
    a2 = fma_v(x2 == T(0) ? T(0) : v2, x2, a2);
    a3 = fma_v(x3 == T(0) ? T(0) : v3, x3, a3);
  }
  for (; j < j1; j++) {
    const T xj = x[j * incx];
    a0 = fma_v(xj == T(0) ? T(0) : a[j * lda], xj, a0);
  }
  const T s = (a0 + a1) + (a2 + a3);
  if (chunks == 1)
    y[i * incy] = finish(s, alpha, beta, y + i * incy);
  else
    partial[(int64_t)blockIdx.y * m + i] = s;
}

// y_i := epilogue(sum over chunks c, in order, of partial[c * len + i]). The
// loads of eight chunks are issued together and then added in chunk order, so
// the sum is the same as a plain loop's but costs one memory round trip per
// eight chunks.
template <typename T>
__global__ void __launch_bounds__(GEMV_THREADS)
    gemv_reduce_kernel(int64_t len, int chunks, const T *__restrict__ partial, T alpha, T beta, T *__restrict__ y,
                       int64_t incy) {
  wg_pdl_wait();     // launched programmatically: the kernel before this one has finished
  wg_pdl_trigger();  // and the next gemv launch may be scheduled
  for (int64_t i = (int64_t)blockIdx.x * GEMV_THREADS + threadIdx.x; i < len;
       i += (int64_t)gridDim.x * GEMV_THREADS) {
    T s = T(0);
    int c = 0;
    for (; c + 8 <= chunks; c += 8) {
      T v[8];
#pragma unroll
      for (int q = 0; q < 8; q++) v[q] = partial[(int64_t)(c + q) * len + i];
#pragma unroll
      for (int q = 0; q < 8; q++) s += v[q];
    }
    for (; c < chunks; c++) s += partial[(int64_t)c * len + i];
    y[i * incy] = finish(s, alpha, beta, y + i * incy);
  }
}

// alpha = 0: y := beta * y (0 when beta = 0, y not read).
template <typename T>
__global__ void __launch_bounds__(GEMV_THREADS) gemv_scale_kernel(int64_t len, T beta, T *__restrict__ y, int64_t incy) {
  wg_pdl_wait();     // launched programmatically: the kernel before this one has finished
  wg_pdl_trigger();  // and the next gemv launch may be scheduled
  for (int64_t i = (int64_t)blockIdx.x * GEMV_THREADS + threadIdx.x; i < len;
       i += (int64_t)gridDim.x * GEMV_THREADS) {
    T *p = y + i * incy;
    *p = beta != T(0) ? beta * *p : T(0);
  }
}

unsigned grid_for(const wg_device *d, int64_t len) {
  const int64_t want = (len + GEMV_THREADS - 1) / GEMV_THREADS;
  const int64_t cap = (int64_t)d->sm_count * 8;  // one element per thread up to 8 CTAs per SM
  return (unsigned)(want < 1 ? 1 : (want < cap ? want : cap));
}

int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Lanes per column segment for gemv_rows_kernel: the widest segment (32, 16, 8
// or 4 lanes of 16 bytes) whose row blocks still give about 0.85 CTAs of 512
// threads per SM (at 4096 rows: 128 CTAs of 32 rows, 128-byte segments, which
// measured faster than more CTAs of narrower segments); 0 = too few rows, so the
// columns are cut into chunks instead (gemv_axpy_vec_kernel and a reduction).
int rows_lanes(const wg_device *d, int64_t m, int64_t vb) {
  const int64_t want = (int64_t)d->sm_count * 85 / 100;
  for (int l = 32; l >= 4; l /= 2)
    if (ceil_div(m, vb * l) >= want) return l;
  return 0;
}

template <typename T, bool UNIT_X>
void launch_rows(int lanes, unsigned g, cudaStream_t s, int64_t m, int64_t n, const T *A, int64_t lda, const T *x,
                 int64_t incx, T alpha, T beta, T *y, int64_t incy) {
  switch (lanes) {
    case 32:
      wg_launch_pdl(gemv_rows_kernel<T, 32, UNIT_X>, dim3(g), dim3(ROWS_THREADS), 0, s, m, n, A, lda, x, incx, alpha,
                    beta, y, incy);
      break;
    case 16:
      wg_launch_pdl(gemv_rows_kernel<T, 16, UNIT_X>, dim3(g), dim3(ROWS_THREADS), 0, s, m, n, A, lda, x, incx, alpha,
                    beta, y, incy);
      break;
    case 8:
      wg_launch_pdl(gemv_rows_kernel<T, 8, UNIT_X>, dim3(g), dim3(ROWS_THREADS), 0, s, m, n, A, lda, x, incx, alpha,
                    beta, y, incy);
      break;
    default:
      wg_launch_pdl(gemv_rows_kernel<T, 4, UNIT_X>, dim3(g), dim3(ROWS_THREADS), 0, s, m, n, A, lda, x, incx, alpha,
                    beta, y, incy);
      break;
  }
}

template <typename T>
wg_status gemv_enqueue(wg_device *d, int trans, int64_t m, int64_t n, T alpha, const T *A, int64_t lda, const T *x,
                       int64_t incx, T beta, T *y, int64_t incy) {
  cudaStream_t s = d->stream;
  const int64_t ylen = trans ? n : m;
  if (alpha == T(0)) {
    wg_launch_scope scope(d, "gemv_scale");
    wg_launch_pdl(gemv_scale_kernel<T>, dim3(grid_for(d, ylen)), dim3(GEMV_THREADS), 0, s, ylen, beta, y, incy);
    WG_CUDA(cudaGetLastError());
    return WG_OK;
  }
  // Loads to keep in flight so that HBM latency is covered.
  const int64_t target = (int64_t)d->sm_count * 2048;
  const size_t vb = 16 / sizeof(T);  // elements of a 16-byte vector
  const bool col_aligned = reinterpret_cast<uintptr_t>(A) % 16 == 0 && lda % (int64_t)vb == 0;
  int64_t chunks = 1, span = 0;
  unsigned gx = 0;
  bool vec = false;
  int64_t mv = 0;  // rows covered by whole vectors (trans = 0)
  int rows_l = 0;  // lanes per column segment of gemv_rows_kernel (trans = 0)
  if (trans) {
    vec = col_aligned && incx == 1 && reinterpret_cast<uintptr_t>(x) % 16 == 0;
    if (vec) {
      // one warp per column: 8 columns per CTA; the rows are cut into chunks only
      // when there are fewer than about 16 columns per SM (each warp keeps 4 KB in flight)
      gx = (unsigned)ceil_div(n, GEMV_THREADS / 32);
      const int64_t warps = (int64_t)gx * (GEMV_THREADS / 32);
      const int64_t want = ceil_div((int64_t)d->sm_count * 16, warps);
      const int64_t most = ceil_div(m, 32 * 8 * (int64_t)vb);  // at least 8 vectors per lane
      chunks = want < most ? want : most;
      if (chunks < 1) chunks = 1;
      span = ceil_div(ceil_div(m, chunks), (int64_t)vb) * (int64_t)vb;
      chunks = ceil_div(m, span);
    } else {
      gx = (unsigned)(n < (int64_t)d->sm_count * 8 ? n : (int64_t)d->sm_count * 8);
      const int64_t want = ceil_div(target, (int64_t)gx * GEMV_THREADS);  // CTAs per column
      const int64_t most = ceil_div(m, 4 * GEMV_THREADS);                  // at least 1024 rows a chunk
      chunks = want < most ? want : most;
      if (chunks < 1) chunks = 1;
      span = ceil_div(m, chunks);
      chunks = ceil_div(m, span);
    }
  } else if (col_aligned && (rows_l = rows_lanes(d, m, (int64_t)vb)) > 0) {
    const int64_t rows = (int64_t)vb * rows_l;
    wg_launch_scope scope(d, "gemv_rows");
    const unsigned g = (unsigned)ceil_div(m, rows);
    if (incx == 1)
      launch_rows<T, true>(rows_l, g, s, m, n, A, lda, x, incx, alpha, beta, y, incy);
    else
      launch_rows<T, false>(rows_l, g, s, m, n, A, lda, x, incx, alpha, beta, y, incy);
    WG_CUDA(cudaGetLastError());
    return WG_OK;
  } else {
    vec = col_aligned && m >= (int64_t)vb;
    mv = vec ? m / (int64_t)vb : 0;
    const int64_t threads = vec ? mv : m;
    const int64_t bx = ceil_div(threads, GEMV_THREADS);
    gx = (unsigned)bx;
    const int64_t per = vec ? 4 : 2;  // 16-byte loads per thread per step count more
    const int64_t want = ceil_div(target / per, bx * GEMV_THREADS);
    const int64_t most = ceil_div(n, 64);  // at least 64 columns a chunk
    chunks = want < most ? want : most;
    if (chunks < 1) chunks = 1;
    if (chunks > 65535) chunks = 65535;
    span = ceil_div(n, chunks);
    chunks = ceil_div(n, span);
  }
  T *partial = nullptr;
  if (chunks > 1) {
    void *ws = nullptr;
    wg_status st = wg_workspace(d, (size_t)chunks * (size_t)ylen * sizeof(T), &ws);
    if (st != WG_OK) return st;
    partial = static_cast<T *>(ws);
  }
  const dim3 grid(gx, (unsigned)chunks);
  if (trans && vec) {
    wg_launch_scope scope(d, "gemv_dot");
    wg_launch_pdl(gemv_dot_vec_kernel<T>, grid, dim3(GEMV_THREADS), 0, s, m, n, A, lda, x, span, (int)chunks, alpha,
                  beta, y, incy, partial);
    WG_CUDA(cudaGetLastError());
  } else if (trans) {
    wg_launch_scope scope(d, "gemv_dot");
    wg_launch_pdl(gemv_dot_kernel<T>, grid, dim3(GEMV_THREADS), 0, s, m, n, A, lda, x, incx, span, (int)chunks, alpha,
                  beta, y, incy, partial);
    WG_CUDA(cudaGetLastError());
  } else {
    wg_launch_scope scope(d, "gemv_axpy");
    if (vec) {
      wg_launch_pdl(gemv_axpy_vec_kernel<T>, grid, dim3(GEMV_THREADS), 0, s, mv, n, A, lda, x, incx, span, (int)chunks,
                    ylen, alpha, beta, y, incy, partial);
      WG_CUDA(cudaGetLastError());
    }
    const int64_t rest = m - mv * (int64_t)vb;  // rows no vector covers
    if (rest > 0) {
      const dim3 g2((unsigned)ceil_div(rest, GEMV_THREADS), (unsigned)chunks);
      wg_launch_pdl(gemv_axpy_kernel<T>, g2, dim3(GEMV_THREADS), 0, s, mv * (int64_t)vb, m, n, A, lda, x, incx, span,
                    (int)chunks, alpha, beta, y, incy, partial);
      WG_CUDA(cudaGetLastError());
    }
  }
  if (chunks > 1) {
    wg_launch_scope scope(d, "gemv_reduce");
    wg_launch_pdl(gemv_reduce_kernel<T>, dim3(grid_for(d, ylen)), dim3(GEMV_THREADS), 0, s, ylen, (int)chunks, partial,
                  alpha, beta, y, incy);
    WG_CUDA(cudaGetLastError());
  }
  return WG_OK;
}

wg_status check_args(wg_device *d, int trans, int64_t m, int64_t n, int64_t lda, int64_t incx, int64_t incy) {
  if (!d) return wg_fail(WG_ERR_INVALID_ARGUMENT, "device is NULL");
  if (trans != 0 && trans != 1)
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "trans must be 0 (no-transpose) or 1 (transpose)");
  if (m < 0 || n < 0) return wg_fail(WG_ERR_INVALID_ARGUMENT, "m and n must be non-negative.");
  if (incx <= 0 || incy <= 0) return wg_fail(WG_ERR_INVALID_ARGUMENT, "incx and incy must be positive.");
  if (lda <= 0) return wg_fail(WG_ERR_INVALID_ARGUMENT, "lda must be positive.");
  const int64_t lim = (int64_t)1 << 31, ld_lim = (int64_t)1 << 40;
  if (m >= lim || n >= lim || lda >= ld_lim || incx >= lim || incy >= lim)
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "dimensions and increments must be below 2^31, lda below 2^40");
  if (m == 0 || n == 0) return WG_OK;
  if (lda < m) return wg_fail(WG_ERR_INVALID_ARGUMENT, "lda must be >= rows of A as stored.");
  if (d->cc_major != 10)
    return wg_fail(WG_ERR_NOT_SUPPORTED, "device %d (%s) is not a Blackwell sm_100 device", d->ordinal, d->name);
  return WG_OK;
}

bool fits_vec(const wg_buffer *b, int64_t off, int64_t len, int64_t inc, size_t elt) {
  if (!b || off < 0) return false;
  const __int128 last = (__int128)off + (__int128)(len - 1) * inc + 1;
  return last * (__int128)elt <= (__int128)b->bytes;
}

bool fits_mat(const wg_buffer *b, int64_t off, int64_t rows, int64_t cols, int64_t ld, size_t elt) {
  if (!b || off < 0) return false;
  const __int128 last = (__int128)off + (__int128)(cols - 1) * ld + rows;
  return last * (__int128)elt <= (__int128)b->bytes;
}

template <typename T>
wg_status gemv_buffers(wg_device *d, int trans, int64_t m, int64_t n, T alpha, const wg_buffer *A, int64_t offA,
                       int64_t lda, const wg_buffer *x, int64_t offx, int64_t incx, T beta, wg_buffer *y,
                       int64_t offy, int64_t incy, float *gpu_ms) {
  if (gpu_ms) *gpu_ms = 0.0f;
  wg_status st = check_args(d, trans, m, n, lda, incx, incy);
  if (st != WG_OK || m == 0 || n == 0) return st;
  if (alpha == T(0) && beta == T(1)) return WG_OK;  // reference BLAS quick return
  const int64_t xlen = trans ? m : n, ylen = trans ? n : m;
  const bool reads = alpha != T(0);
  if (!fits_vec(y, offy, ylen, incy, sizeof(T)))
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "y does not have enough elements for the given dimensions and incy.");
  if (reads && !fits_vec(x, offx, xlen, incx, sizeof(T)))
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "x does not have enough elements for the given dimensions and incx.");
  if (reads && !fits_mat(A, offA, m, n, lda, sizeof(T)))
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "A does not have enough elements for the given m, n, and lda.");
  if (y->dev->ordinal != d->ordinal || (reads && (A->dev->ordinal != d->ordinal || x->dev->ordinal != d->ordinal)))
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "a buffer belongs to another device");
  wg_device_guard guard(d->ordinal);
  const bool timing = gpu_ms && (d->flags & WG_DEVICE_TIMING);
  if (timing) WG_CUDA(cudaEventRecord(d->ev_start, d->stream));
  st = gemv_enqueue<T>(d, trans, m, n, alpha, reads ? static_cast<const T *>(A->ptr) + offA : nullptr, lda,
                       reads ? static_cast<const T *>(x->ptr) + offx : nullptr, incx, beta,
                       static_cast<T *>(y->ptr) + offy, incy);
  if (st != WG_OK) return st;
  if (timing) {
    WG_CUDA(cudaEventRecord(d->ev_stop, d->stream));
    WG_CUDA(cudaEventSynchronize(d->ev_stop));
    WG_CUDA(cudaEventElapsedTime(gpu_ms, d->ev_start, d->ev_stop));
  }
  return WG_OK;
}

template <typename T>
wg_status gemv_dev(wg_device *d, int trans, int64_t m, int64_t n, T alpha, const T *A, int64_t lda, const T *x,
                   int64_t incx, T beta, T *y, int64_t incy) {
  wg_status st = check_args(d, trans, m, n, lda, incx, incy);
  if (st != WG_OK || m == 0 || n == 0 || (alpha == T(0) && beta == T(1))) return st;
  if (!y || (alpha != T(0) && (!A || !x))) return wg_fail(WG_ERR_INVALID_ARGUMENT, "operand pointer is NULL");
  wg_device_guard guard(d->ordinal);
  return gemv_enqueue<T>(d, trans, m, n, alpha, A, lda, x, incx, beta, y, incy);
}

}  // namespace

extern "C" wg_status wg_sgemv(wg_device *d, int trans, int64_t m, int64_t n, float alpha, const wg_buffer *A,
                              int64_t offA, int64_t lda, const wg_buffer *x, int64_t offx, int64_t incx, float beta,
                              wg_buffer *y, int64_t offy, int64_t incy, float *gpu_ms) {
  return gemv_buffers<float>(d, trans, m, n, alpha, A, offA, lda, x, offx, incx, beta, y, offy, incy, gpu_ms);
}

extern "C" wg_status wg_dgemv(wg_device *d, int trans, int64_t m, int64_t n, double alpha, const wg_buffer *A,
                              int64_t offA, int64_t lda, const wg_buffer *x, int64_t offx, int64_t incx, double beta,
                              wg_buffer *y, int64_t offy, int64_t incy, float *gpu_ms) {
  return gemv_buffers<double>(d, trans, m, n, alpha, A, offA, lda, x, offx, incx, beta, y, offy, incy, gpu_ms);
}

extern "C" wg_status wg_sgemv_dev(wg_device *d, int trans, int64_t m, int64_t n, float alpha, const float *A,
                                  int64_t lda, const float *x, int64_t incx, float beta, float *y, int64_t incy) {
  return gemv_dev<float>(d, trans, m, n, alpha, A, lda, x, incx, beta, y, incy);
}

extern "C" wg_status wg_dgemv_dev(wg_device *d, int trans, int64_t m, int64_t n, double alpha, const double *A,
                                  int64_t lda, const double *x, int64_t incx, double beta, double *y, int64_t incy) {
  return gemv_dev<double>(d, trans, m, n, alpha, A, lda, x, incx, beta, y, incy);
}
