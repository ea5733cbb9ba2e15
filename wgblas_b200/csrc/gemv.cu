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

// trans = 0. Columns [c * cols, min(n, (c + 1) * cols)) of chunk c = blockIdx.y.
template <typename T>
__global__ void __launch_bounds__(GEMV_THREADS)
    gemv_axpy_kernel(int64_t m, int64_t n, const T *__restrict__ A, int64_t lda, const T *__restrict__ x,
                     int64_t incx, int64_t cols, int chunks, T alpha, T beta, T *__restrict__ y, int64_t incy,
                     T *__restrict__ partial) {
  const int64_t i = (int64_t)blockIdx.x * GEMV_THREADS + threadIdx.x;
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

// y_i := epilogue(sum over chunks c, in order, of partial[c * len + i]).
template <typename T>
__global__ void __launch_bounds__(GEMV_THREADS)
    gemv_reduce_kernel(int64_t len, int chunks, const T *__restrict__ partial, T alpha, T beta, T *__restrict__ y,
                       int64_t incy) {
  for (int64_t i = (int64_t)blockIdx.x * GEMV_THREADS + threadIdx.x; i < len;
       i += (int64_t)gridDim.x * GEMV_THREADS) {
    T s = T(0);
    for (int c = 0; c < chunks; c++) s += partial[(int64_t)c * len + i];
    y[i * incy] = finish(s, alpha, beta, y + i * incy);
  }
}

// alpha = 0: y := beta * y (0 when beta = 0, y not read).
template <typename T>
__global__ void __launch_bounds__(GEMV_THREADS) gemv_scale_kernel(int64_t len, T beta, T *__restrict__ y, int64_t incy) {
  for (int64_t i = (int64_t)blockIdx.x * GEMV_THREADS + threadIdx.x; i < len;
       i += (int64_t)gridDim.x * GEMV_THREADS) {
    T *p = y + i * incy;
    *p = beta != T(0) ? beta * *p : T(0);
  }
}

unsigned grid_for(const wg_device *d, int64_t len) {
  const int64_t want = (len + GEMV_THREADS - 1) / GEMV_THREADS;
  const int64_t cap = (int64_t)d->sm_count * 8;
  return (unsigned)(want < 1 ? 1 : (want < cap ? want : cap));
}

int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

template <typename T>
wg_status gemv_enqueue(wg_device *d, int trans, int64_t m, int64_t n, T alpha, const T *A, int64_t lda, const T *x,
                       int64_t incx, T beta, T *y, int64_t incy) {
  cudaStream_t s = d->stream;
  const int64_t ylen = trans ? n : m;
  if (alpha == T(0)) {
    wg_launch_scope scope(d, "gemv_scale");
    gemv_scale_kernel<T><<<grid_for(d, ylen), GEMV_THREADS, 0, s>>>(ylen, beta, y, incy);
    WG_CUDA(cudaGetLastError());
    return WG_OK;
  }
  // Threads to keep in flight so that HBM latency is covered: about 2048 per SM.
  const int64_t target = (int64_t)d->sm_count * 2048;
  int64_t chunks = 1, span = 0;
  unsigned gx = 0;
  if (trans) {
    gx = (unsigned)(n < (int64_t)d->sm_count * 8 ? n : (int64_t)d->sm_count * 8);
    const int64_t want = ceil_div(target, (int64_t)gx * GEMV_THREADS);  // CTAs per column
    const int64_t most = ceil_div(m, 4 * GEMV_THREADS);                  // at least 1024 rows a chunk
    chunks = want < most ? want : most;
    if (chunks < 1) chunks = 1;
    span = ceil_div(m, chunks);
    chunks = ceil_div(m, span);
  } else {
    const int64_t bx = ceil_div(m, GEMV_THREADS);
    gx = (unsigned)bx;
    const int64_t want = ceil_div(target, bx * GEMV_THREADS);
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
  if (trans) {
    wg_launch_scope scope(d, "gemv_dot");
    gemv_dot_kernel<T><<<grid, GEMV_THREADS, 0, s>>>(m, n, A, lda, x, incx, span, (int)chunks, alpha, beta, y, incy,
                                                     partial);
    WG_CUDA(cudaGetLastError());
  } else {
    wg_launch_scope scope(d, "gemv_axpy");
    gemv_axpy_kernel<T><<<grid, GEMV_THREADS, 0, s>>>(m, n, A, lda, x, incx, span, (int)chunks, alpha, beta, y,
                                                      incy, partial);
    WG_CUDA(cudaGetLastError());
  }
  if (chunks > 1) {
    wg_launch_scope scope(d, "gemv_reduce");
    gemv_reduce_kernel<T><<<grid_for(d, ylen), GEMV_THREADS, 0, s>>>(ylen, (int)chunks, partial, alpha, beta, y,
                                                                     incy);
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
