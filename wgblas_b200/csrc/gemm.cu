// sgemm / dgemm entry points of the C ABI: argument checks, kernel choice,
// event timing and the host-array path.
//
// Replaces the dispatch half of src/sgemm/sgemm.mjs:25-269 and
// src/dgemm/dgemm.mjs:23-318 (tile selection, upload, one compute pass,
// readback). Argument-shape errors that the JavaScript layer reports with its
// own messages (src/sgemm/sgemm.mjs:46-149) are re-checked here in the
// column-major frame so that a C caller gets WG_ERR_INVALID_ARGUMENT instead of
// an out-of-bounds access.
#include <cstring>
#include <type_traits>
#include <vector>

#include "internal.h"

namespace {

// Rows and columns of the stored matrix behind op(X) (column-major frame).
struct Stored {
  int64_t rows, cols;
};

bool fits(int64_t off, int64_t ld, Stored s, size_t elems) {
  if (s.rows == 0 || s.cols == 0) return off >= 0 && (unsigned __int128)off <= elems;
  __int128 last = (__int128)off + (__int128)(s.cols - 1) * ld + s.rows;
  return off >= 0 && last <= (__int128)elems;
}

wg_status check_dims(int transA, int transB, int64_t m, int64_t n, int64_t k, int64_t lda,
                     int64_t ldb, int64_t ldc) {
  if ((transA != 0 && transA != 1) || (transB != 0 && transB != 1))
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "transA and transB must be 0 (no-transpose) or 1 (transpose)");
  if (m < 0 || n < 0 || k < 0) return wg_fail(WG_ERR_INVALID_ARGUMENT, "m, n, and k must be non-negative.");
  if (lda <= 0 || ldb <= 0 || ldc <= 0)
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "lda, ldb, and ldc must be positive.");
  const int64_t lim = (int64_t)1 << 31;
  if (m >= lim || n >= lim || k >= lim || lda >= ((int64_t)1 << 40) || ldb >= ((int64_t)1 << 40) ||
      ldc >= ((int64_t)1 << 40))
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "dimensions must be below 2^31 and leading dimensions below 2^40");
  if (lda < (transA ? k : m))
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "lda must be >= rows of A as stored.");
  if (ldb < (transB ? n : k))
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "ldb must be >= rows of B as stored.");
  if (ldc < m) return wg_fail(WG_ERR_INVALID_ARGUMENT, "ldc must be >= rows of C as stored.");
  return WG_OK;
}

Stored stored_a(int transA, int64_t m, int64_t k) { return transA ? Stored{k, m} : Stored{m, k}; }
Stored stored_b(int transB, int64_t n, int64_t k) { return transB ? Stored{n, k} : Stored{k, n}; }

// Whether the device can run the sm_100a kernels in this library at all.
wg_status check_arch(const wg_device *d) {
  if (d->cc_major != 10)
    return wg_fail(WG_ERR_NOT_SUPPORTED,
                   "device %d (%s, sm_%d%d) is not a Blackwell sm_100 device; this library is built "
                   "for sm_100a only", d->ordinal, d->name, d->cc_major, d->cc_minor);
  return WG_OK;
}

template <typename T>
wg_status gemm_launch(wg_device *d, int transA, int transB, int64_t m, int64_t n, int64_t k, T alpha,
                      const T *A, int64_t lda, const T *B, int64_t ldb, T beta, T *C, int64_t ldc, int uplo = 0);
}  // namespace

template <typename T>
wg_status wg_gemm_enqueue(wg_device *d, int transA, int transB, int64_t m, int64_t n, int64_t k, T alpha,
                          const T *A, int64_t lda, const T *B, int64_t ldb, T beta, T *C, int64_t ldc, int uplo) {
  if (m == 0 || n == 0) return WG_OK;
  return gemm_launch<T>(d, transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, uplo);
}

namespace {

// Small products on the FFMA pipe: the 32 x 64-tile kernel beats the 3xTF32
// kernels while its tiles take at most two waves over the SMs and each SM runs
// at most 80 of its 16-deep k-tiles. Measured per call on B200 with L2 flushed
// between calls: 256^3 22 vs 38 us, 512^3 28 vs 41 us, 640^3 43 vs 45 us,
// 64 x 4096 x 64 8.8 vs 13.3 us; 768^3 51 vs 47 us, 256 x 256 x 4096 127 vs
// 57 us and 256 x 4096 x 256 (four waves) 33.6 vs 19.3 us go to the tensor cores.
bool small_ffma_wins(const wg_device *d, int64_t m, int64_t n, int64_t k) {
  const int64_t tiles = ((m + 31) / 32) * ((n + 63) / 64), sm = d->sm_count > 0 ? d->sm_count : 1;
  const int64_t waves = (tiles + sm - 1) / sm;
  return waves <= 2 && waves * ((k + 15) / 16) <= 80;
}

// FFMA work (no tensor cores) goes to the 32 x 64-tile kernel when asked, when
// it is a small product (above), or when the 128 x 128-tile kernel would not
// have a tile for every SM.
bool simt_small_tiles(const wg_device *d, int path, int64_t m, int64_t n, int64_t k) {
  if (path == WG_SGEMM_SIMT_SMALL) return true;
  return path == WG_SGEMM_AUTO &&
         (small_ffma_wins(d, m, n, k) || ((m + 127) / 128) * ((n + 127) / 128) < d->sm_count);
}

// sgemm kernel choice. The 3xTF32 tensor-core kernel needs enough k to amortise
// its split pass and gives no benefit on tiny grids or small products (above);
// everything else, and any call whose operands fail the split's range check on
// the device, runs an FFMA kernel.
template <>
wg_status gemm_launch<float>(wg_device *d, int transA, int transB, int64_t m, int64_t n, int64_t k,
                             float alpha, const float *A, int64_t lda, const float *B, int64_t ldb,
                             float beta, float *C, int64_t ldc, int uplo) {
  cudaStream_t s = d->stream;
  if (alpha == 0.0f || k == 0) {
    wg_launch_scope scope(d, "scale");
    WG_CUDA(wg_launch_scale<float>(s, m, n, alpha, beta, C, ldc, uplo));
    return WG_OK;
  }
  d->stats.calls++;
  bool tc = false;
  const int path = d->sgemm_path;
  const bool forced_tc = path >= WG_SGEMM_TF32X3 && path <= WG_SGEMM_TF32X3_PAIR;
  if (forced_tc) {
    if (!wg_tf32x3_supported(d, m, n, k))
      return wg_fail(WG_ERR_NOT_SUPPORTED, "the 3xTF32 kernel does not support m=%lld n=%lld k=%lld",
                     (long long)m, (long long)n, (long long)k);
    tc = true;
  } else if (path == WG_SGEMM_AUTO) {
    tc = wg_tf32x3_supported(d, m, n, k) && k >= 64 && (double)m * (double)n >= 256.0 * 256.0 &&
         !small_ffma_wins(d, m, n, k);
  }
  const bool aligned = tc && path != WG_SGEMM_TF32X3_PACKED &&
                       wg_tf32x3_fused_supported(d, transA, transB, m, n, k, A, lda, B, ldb);
  const bool small = (double)m * (double)n * (double)k <= WG_FUSED_MAX_WORK;
  const bool forced_fused = path >= WG_SGEMM_TF32X3_FUSED_BN256 && path <= WG_SGEMM_TF32X3_FUSED_BN64;
  // Above WG_FUSED_MAX_WORK the split pass + MMA kernel is the faster path (the
  // in-kernel split of either fused form is latency-bound there); the pair form
  // runs only when asked for.
  const bool pair = aligned && path == WG_SGEMM_TF32X3_PAIR;
  const bool fused = aligned && !pair && (forced_fused || small);
  if ((forced_fused || path == WG_SGEMM_TF32X3_PAIR) && !aligned)
    return wg_fail(WG_ERR_NOT_SUPPORTED, "the fused 3xTF32 kernel needs 16-byte aligned A and B and lda, ldb "
                   "multiples of 4");
  if (pair) {
    void *ws = nullptr;
    const size_t bytes = wg_tf32x3_pair_workspace(d, m, n, k);
    wg_status st = wg_workspace(d, bytes, &ws);
    if (st != WG_OK) return st;
    st = wg_sgemm_tf32x3_pair(d, d->stream, transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, ws, bytes,
                              uplo);
    if (st != WG_OK) return st;
    d->stats.tf32x3_launches++;
    return WG_OK;
  }
  if (fused) {
    void *ws = nullptr;
    const size_t bytes = wg_tf32x3_fused_workspace(d, m, n, k);
    wg_status st = wg_workspace(d, bytes, &ws);
    if (st != WG_OK) return st;
    st = wg_sgemm_tf32x3_fused(d, d->stream, transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, ws,
                               bytes, uplo);
    if (st != WG_OK) return st;
    d->stats.tf32x3_launches++;
    return WG_OK;
  }
  if (tc) {
    void *ws = nullptr;
    const size_t bytes = wg_tf32x3_workspace_bytes_sk(d, m, n, k);
    wg_status st = wg_workspace(d, bytes, &ws);
    if (st != WG_OK) return st;
    st = wg_sgemm_tf32x3(d, transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, ws, bytes, uplo);
    if (st != WG_OK) return st;
    d->stats.tf32x3_launches++;
    return WG_OK;
  }
  d->stats.simt_launches++;
  if (simt_small_tiles(d, path, m, n, k)) {
    wg_launch_scope scope(d, "sgemm_simt_small");
    WG_CUDA(wg_launch_gemm_simt_small(s, transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, uplo));
    return WG_OK;
  }
  wg_launch_scope scope(d, "sgemm_simt");
  WG_CUDA(wg_launch_gemm_simt<float>(s, transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc,
                                     d->dwords, nullptr, uplo));
  return WG_OK;
}

template <>
wg_status gemm_launch<double>(wg_device *d, int transA, int transB, int64_t m, int64_t n, int64_t k,
                              double alpha, const double *A, int64_t lda, const double *B,
                              int64_t ldb, double beta, double *C, int64_t ldc, int uplo) {
  cudaStream_t s = d->stream;
  if (alpha == 0.0 || k == 0) {
    wg_launch_scope scope(d, "scale");
    WG_CUDA(wg_launch_scale<double>(s, m, n, alpha, beta, C, ldc, uplo));
    return WG_OK;
  }
  // The DMMA kernel needs a few k steps and a grid worth filling; small calls run
  // the DFMA kernel, whose sequential FMA chains match the CPU restatement bit for bit.
  const bool dmma = d->dgemm_path == WG_DGEMM_DMMA ||
                    (d->dgemm_path == WG_DGEMM_AUTO && k >= 16 && (double)m * (double)n >= 128.0 * 128.0);
  if (dmma) return wg_dgemm_dmma(d, transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, uplo);
  wg_launch_scope scope(d, "dgemm_simt");
  WG_CUDA(wg_launch_gemm_simt<double>(s, transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C,
                                      ldc, d->dwords, nullptr, uplo));
  return WG_OK;
}

// dgemm's quick return (src/dgemm/dgemm.mjs:177-179); sgemm has none.
template <typename T>
bool quick_return(int64_t k, T alpha, T beta);
template <>
bool quick_return<float>(int64_t, float, float) { return false; }
template <>
bool quick_return<double>(int64_t k, double alpha, double beta) {
  return (alpha == 0.0 || k == 0) && beta == 1.0;
}

template <typename T>
wg_status gemm_timed(wg_device *d, int transA, int transB, int64_t m, int64_t n, int64_t k, T alpha,
                     const T *A, int64_t lda, const T *B, int64_t ldb, T beta, T *C, int64_t ldc,
                     float *gpu_ms, int uplo) {
  const bool timing = gpu_ms && (d->flags & WG_DEVICE_TIMING);
  if (timing) WG_CUDA(cudaEventRecord(d->ev_start, d->stream));
  wg_status st = gemm_launch<T>(d, transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, uplo);
  if (st != WG_OK) return st;
  if (timing) {
    WG_CUDA(cudaEventRecord(d->ev_stop, d->stream));
    WG_CUDA(cudaEventSynchronize(d->ev_stop));
    WG_CUDA(cudaEventElapsedTime(gpu_ms, d->ev_start, d->ev_stop));
  }
  return WG_OK;
}

template <typename T>
wg_status gemm_buffers(wg_device *d, int transA, int transB, int64_t m, int64_t n, int64_t k, T alpha,
                       const wg_buffer *A, int64_t offA, int64_t lda, const wg_buffer *B, int64_t offB,
                       int64_t ldb, T beta, wg_buffer *C, int64_t offC, int64_t ldc, float *gpu_ms,
                       int uplo = WG_UPLO_FULL) {
  if (gpu_ms) *gpu_ms = 0.0f;
  if (!d) return wg_fail(WG_ERR_INVALID_ARGUMENT, "device is NULL");
  if (uplo < WG_UPLO_FULL || uplo > WG_UPLO_UPPER)
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "uplo must be 'lower' or 'upper'.");
  wg_status st = check_dims(transA, transB, m, n, k, lda, ldb, ldc);
  if (st != WG_OK) return st;
  if (m == 0 || n == 0) return WG_OK;  // src/sgemm/sgemm.mjs:83
  if (quick_return<T>(k, alpha, beta)) return WG_OK;
  if (!A || !B || !C) return wg_fail(WG_ERR_INVALID_ARGUMENT, "A, B and C must be buffers");
  for (const wg_buffer *b : {A, B, (const wg_buffer *)C})
    if (b->dev->ordinal != d->ordinal)
      return wg_fail(WG_ERR_INVALID_ARGUMENT,
                     "a buffer belongs to device %d, not to device %d that the call runs on",
                     b->dev->ordinal, d->ordinal);
  const bool reads_ab = k > 0 && alpha != T(0);
  if (reads_ab && !fits(offA, lda, stored_a(transA, m, k), A->bytes / sizeof(T)))
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "A does not have enough elements for the given dimensions and lda.");
  if (reads_ab && !fits(offB, ldb, stored_b(transB, n, k), B->bytes / sizeof(T)))
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "B does not have enough elements for the given dimensions and ldb.");
  if (!fits(offC, ldc, Stored{m, n}, C->bytes / sizeof(T)))
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "C does not have enough elements for the given dimensions and ldc.");
  st = check_arch(d);
  if (st != WG_OK) return st;
  wg_device_guard guard(d->ordinal);
  return gemm_timed<T>(d, transA, transB, m, n, k, alpha, (const T *)A->ptr + offA, lda,
                       (const T *)B->ptr + offB, ldb, beta, (T *)C->ptr + offC, ldc, gpu_ms, uplo);
}

template <typename T>
wg_status gemm_dev(wg_device *d, int transA, int transB, int64_t m, int64_t n, int64_t k, T alpha,
                   const T *A, int64_t lda, const T *B, int64_t ldb, T beta, T *C, int64_t ldc,
                   int uplo = WG_UPLO_FULL) {
  if (!d) return wg_fail(WG_ERR_INVALID_ARGUMENT, "device is NULL");
  if (uplo < WG_UPLO_FULL || uplo > WG_UPLO_UPPER)
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "uplo must be 'lower' or 'upper'.");
  wg_status st = check_dims(transA, transB, m, n, k, lda, ldb, ldc);
  if (st != WG_OK) return st;
  if (m == 0 || n == 0 || quick_return<T>(k, alpha, beta)) return WG_OK;
  if ((k > 0 && alpha != T(0) && (!A || !B)) || !C)
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "operand pointer is NULL");
  st = check_arch(d);
  if (st != WG_OK) return st;
  wg_device_guard guard(d->ordinal);
  return gemm_launch<T>(d, transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, uplo);
}

// Copies the rows x cols block of a column-major host matrix (leading dimension
// ld) into a device matrix with leading dimension dst_ld (>= rows).
template <typename T>
cudaError_t h2d_block(T *dst, int64_t dst_ld, const T *src, int64_t ld, Stored s, cudaStream_t st) {
  if (s.rows == 0 || s.cols == 0) return cudaSuccess;
  return cudaMemcpy2DAsync(dst, dst_ld * sizeof(T), src, ld * sizeof(T), s.rows * sizeof(T), s.cols,
                           cudaMemcpyHostToDevice, st);
}

// Leading dimension of a device copy: rows rounded up to 4 elements, so that
// every column starts on a 16-byte boundary (the TMA-fed kernels' requirement).
int64_t device_ld(int64_t rows) { return rows > 0 ? (rows + 3) / 4 * 4 : 4; }

// Panel width of the host-array path: wide enough that each panel's GEMM is
// efficient, narrow enough that the upload, the GEMM and the read-back of
// consecutive panels overlap.
int64_t host_panel_cols(int64_t m, int64_t n, int64_t k) {
  const double flops = 2.0 * (double)m * (double)n * (double)k;
  if (flops < 2e9 || n < 512) return n;  // too small to be worth splitting
  int64_t p = (n + 3) / 4;
  p = (p + 255) / 256 * 256;
  return p < n ? p : n;
}

struct HostPipe {
  cudaEvent_t ev_a = nullptr;  // op(A) on the device
  std::vector<cudaEvent_t> ev_b, ev_c;
  ~HostPipe() {
    if (ev_a) cudaEventDestroy(ev_a);
    for (cudaEvent_t e : ev_b) cudaEventDestroy(e);
    for (cudaEvent_t e : ev_c) cudaEventDestroy(e);
  }
};

// The typed-array path: op(A) is uploaded once; op(B) (and C when beta != 0)
// is uploaded in column panels on a copy stream, each panel's GEMM starts when
// its panel has arrived, and each finished panel of C is read back on a second
// copy stream while the next one uploads and computes. Page-locked host arrays
// make all three overlap.
template <typename T>
wg_status gemm_host(wg_device *d, int transA, int transB, int64_t m, int64_t n, int64_t k, T alpha,
                    const T *A, int64_t lda, const T *B, int64_t ldb, T beta, const T *C_in, T *C_out,
                    int64_t ldc, float *gpu_ms, int uplo = WG_UPLO_FULL) {
  if (gpu_ms) *gpu_ms = 0.0f;
  if (!d) return wg_fail(WG_ERR_INVALID_ARGUMENT, "device is NULL");
  if (uplo < WG_UPLO_FULL || uplo > WG_UPLO_UPPER)
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "uplo must be 'lower' or 'upper'.");
  wg_status st = check_dims(transA, transB, m, n, k, lda, ldb, ldc);
  if (st != WG_OK) return st;
  if (!C_out) return wg_fail(WG_ERR_INVALID_ARGUMENT, "C_out is NULL");
  if (m == 0 || n == 0) return WG_OK;
  const bool reads_ab = k > 0 && alpha != T(0);
  // gemmtr leaves C outside the triangle as it came in, so C always goes up.
  const bool reads_c = beta != T(0) || uplo != WG_UPLO_FULL;
  if ((reads_ab && (!A || !B)) || (reads_c && !C_in))
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "operand pointer is NULL");
  if (quick_return<T>(k, alpha, beta)) {
    // C is returned as it came in (src/dgemm/dgemm.mjs:179).
    if (C_out != C_in)
      for (int64_t j = 0; j < n; j++) memcpy(C_out + j * ldc, C_in + j * ldc, m * sizeof(T));
    return WG_OK;
  }
  st = check_arch(d);
  if (st != WG_OK) return st;
  wg_device_guard guard(d->ordinal);
  if (!d->h2d) WG_CUDA(cudaStreamCreateWithFlags(&d->h2d, cudaStreamNonBlocking));
  if (!d->d2h) WG_CUDA(cudaStreamCreateWithFlags(&d->d2h, cudaStreamNonBlocking));
  st = wg_staging_pool(d);
  if (st != WG_OK) return st;
  cudaStream_t s = d->stream;
  const Stored sa = stored_a(transA, m, k), sb = stored_b(transB, n, k);
  const int64_t lda_d = device_ld(sa.rows), ldb_d = device_ld(sb.rows);
  const size_t na = reads_ab ? (size_t)(lda_d * sa.cols) : 0;
  const size_t nb = reads_ab ? (size_t)(ldb_d * sb.cols) : 0;
  const size_t nc = (size_t)(m * n);
  const int64_t panel = reads_ab && uplo == WG_UPLO_FULL ? host_panel_cols(m, n, k) : n;
  const int64_t panels = (n + panel - 1) / panel;
  // sgemm panels on the tensor cores run as one wg_tc_product, whose op(B)
  // splits overlap the previous panel's MMA.
  // A small product as a whole (small_ffma_wins) keeps its panels on the FFMA kernel.
  const bool tc = panels > 1 && std::is_same<T, float>::value && wg_sgemm_panel_on_tc(d, (float)alpha, m, panel, k) &&
                  !(d->sgemm_path == WG_SGEMM_AUTO && small_ffma_wins(d, m, n, k));
  const int64_t widths[2] = {panel, n - (panels - 1) * panel};
  wg_tc_product prod{};
  HostPipe pipe;
  T *dA = nullptr, *dB = nullptr, *dC = nullptr;
  cudaError_t e = cudaSuccess;
  // Stream-ordered temporaries, released in stream order like the reference's
  // `finally` (src/sgemm/sgemm.mjs:263-268); the pool keeps the memory mapped
  // for the next call.
  e = cudaMallocFromPoolAsync((void **)&dC, nc * sizeof(T), d->staging, s);
  if (e == cudaSuccess && na) e = cudaMallocFromPoolAsync((void **)&dA, na * sizeof(T), d->staging, s);
  if (e == cudaSuccess && nb) e = cudaMallocFromPoolAsync((void **)&dB, nb * sizeof(T), d->staging, s);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&pipe.ev_a, cudaEventDisableTiming);
  for (int64_t j = 0; e == cudaSuccess && j < panels; j++) {
    cudaEvent_t eb = nullptr, ec = nullptr;
    e = cudaEventCreateWithFlags(&eb, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ec, cudaEventDisableTiming);
    pipe.ev_b.push_back(eb);
    pipe.ev_c.push_back(ec);
  }
  // The copy streams start after the allocations (made on the compute stream).
  if (e == cudaSuccess) e = cudaEventRecord(pipe.ev_a, s);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(d->h2d, pipe.ev_a, 0);
  if (e == cudaSuccess && na) e = h2d_block(dA, lda_d, A, lda, sa, d->h2d);
  if (e == cudaSuccess) e = cudaEventRecord(pipe.ev_a, d->h2d);
  for (int64_t j = 0; e == cudaSuccess && j < panels; j++) {
    const int64_t j0 = j * panel, cols = n - j0 < panel ? n - j0 : panel;
    if (nb) {
      if (transB)  // rows j0.. of the n x k stored B
        e = cudaMemcpy2DAsync(dB + j0, ldb_d * sizeof(T), B + j0, ldb * sizeof(T), cols * sizeof(T), k,
                              cudaMemcpyHostToDevice, d->h2d);
      else         // columns j0.. of the k x n stored B
        e = h2d_block(dB + j0 * ldb_d, ldb_d, B + j0 * ldb, ldb, Stored{k, cols}, d->h2d);
    }
    if (e == cudaSuccess && reads_c)
      e = h2d_block(dC + j0 * m, m, C_in + j0 * ldc, ldc, Stored{m, cols}, d->h2d);
    if (e == cudaSuccess) e = cudaEventRecord(pipe.ev_b[j], d->h2d);
  }
  const bool timing = gpu_ms && (d->flags & WG_DEVICE_TIMING);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(s, pipe.ev_a, 0);
  if (e == cudaSuccess && timing) e = cudaEventRecord(d->ev_start, s);
  if (e == cudaSuccess && tc)
    st = wg_tc_product_begin(&prod, d, transA, transB, m, k, (float)alpha, (const float *)dA, lda_d, (float)beta,
                             widths, 2, pipe.ev_a, (const float *)dB, ldb_d);
  for (int64_t j = 0; e == cudaSuccess && st == WG_OK && j < panels; j++) {
    const int64_t j0 = j * panel, cols = n - j0 < panel ? n - j0 : panel;
    const T *bp = dB ? (transB ? dB + j0 : dB + j0 * ldb_d) : nullptr;
    if (tc) {
      st = wg_tc_product_panel(&prod, cols, (const float *)bp, ldb_d, (float *)(dC + j0 * m), m, pipe.ev_b[j]);
    } else {
      e = cudaStreamWaitEvent(s, pipe.ev_b[j], 0);
      if (e != cudaSuccess) break;
      st = panels == 1 ? gemm_launch<T>(d, transA, transB, m, cols, k, alpha, dA, lda_d, bp, ldb_d, beta, dC, m, uplo)
                       : wg_gemm_panel<T>(d, transA, transB, m, cols, k, alpha, dA, lda_d, bp, ldb_d, beta,
                                          dC + j0 * m, m);
    }
    if (st != WG_OK) break;
    e = cudaEventRecord(pipe.ev_c[j], s);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(d->d2h, pipe.ev_c[j], 0);
    if (e == cudaSuccess)
      e = cudaMemcpy2DAsync(C_out + j0 * ldc, ldc * sizeof(T), dC + j0 * m, m * sizeof(T), m * sizeof(T), cols,
                            cudaMemcpyDeviceToHost, d->d2h);
  }
  if (e == cudaSuccess && st == WG_OK && timing) e = cudaEventRecord(d->ev_stop, s);
  if (tc) wg_tc_product_join(&prod);
  // The temporaries are released once the last read-back has finished.
  cudaEvent_t done = panels ? pipe.ev_c[panels - 1] : pipe.ev_a;
  if (cudaEventRecord(done, d->d2h) == cudaSuccess) cudaStreamWaitEvent(s, done, 0);
  if (dA) cudaFreeAsync(dA, s);
  if (dB) cudaFreeAsync(dB, s);
  if (dC) cudaFreeAsync(dC, s);
  cudaError_t e2 = cudaStreamSynchronize(s);
  if (st != WG_OK) return st;
  if (e == cudaSuccess) e = e2;
  if (e == cudaSuccess && timing) e = cudaEventElapsedTime(gpu_ms, d->ev_start, d->ev_stop);
  if (e != cudaSuccess)
    return wg_fail(e == cudaErrorMemoryAllocation ? WG_ERR_OUT_OF_MEMORY : WG_ERR_CUDA,
                   "host-array GEMM failed: %s", cudaGetErrorString(e));
  return WG_OK;
}

}  // namespace

template <typename T>
wg_status wg_gemm_panel(wg_device *d, int transA, int transB, int64_t m, int64_t cols, int64_t k, T alpha,
                        const T *A, int64_t lda, const T *B, int64_t ldb, T beta, T *C, int64_t ldc) {
  return wg_gemm_enqueue<T>(d, transA, transB, m, cols, k, alpha, A, lda, B, ldb, beta, C, ldc);
}

bool wg_sgemm_panel_on_tc(const wg_device *d, float alpha, int64_t m, int64_t cols, int64_t k) {
  return d->sgemm_path != WG_SGEMM_SIMT && d->sgemm_path != WG_SGEMM_SIMT_SMALL && alpha != 0.0f && k >= 64 &&
         m > 0 && cols > 0 &&
         wg_tf32x3_supported(d, m, cols, k);
}

template wg_status wg_gemm_panel<float>(wg_device *, int, int, int64_t, int64_t, int64_t, float, const float *,
                                        int64_t, const float *, int64_t, float, float *, int64_t);
template wg_status wg_gemm_panel<double>(wg_device *, int, int, int64_t, int64_t, int64_t, double, const double *,
                                         int64_t, const double *, int64_t, double, double *, int64_t);

template wg_status wg_gemm_enqueue<float>(wg_device *, int, int, int64_t, int64_t, int64_t, float, const float *,
                                          int64_t, const float *, int64_t, float, float *, int64_t, int);
template wg_status wg_gemm_enqueue<double>(wg_device *, int, int, int64_t, int64_t, int64_t, double,
                                           const double *, int64_t, const double *, int64_t, double, double *,
                                           int64_t, int);

extern "C" wg_status wg_sgemm(wg_device *d, int transA, int transB, int64_t m, int64_t n, int64_t k,
                              float alpha, const wg_buffer *A, int64_t offA, int64_t lda,
                              const wg_buffer *B, int64_t offB, int64_t ldb, float beta, wg_buffer *C,
                              int64_t offC, int64_t ldc, float *gpu_ms) {
  return gemm_buffers<float>(d, transA, transB, m, n, k, alpha, A, offA, lda, B, offB, ldb, beta, C,
                             offC, ldc, gpu_ms);
}

extern "C" wg_status wg_dgemm(wg_device *d, int transA, int transB, int64_t m, int64_t n, int64_t k,
                              double alpha, const wg_buffer *A, int64_t offA, int64_t lda,
                              const wg_buffer *B, int64_t offB, int64_t ldb, double beta, wg_buffer *C,
                              int64_t offC, int64_t ldc, float *gpu_ms) {
  return gemm_buffers<double>(d, transA, transB, m, n, k, alpha, A, offA, lda, B, offB, ldb, beta, C,
                              offC, ldc, gpu_ms);
}

extern "C" wg_status wg_sgemm_dev(wg_device *d, int transA, int transB, int64_t m, int64_t n, int64_t k,
                                  float alpha, const float *A, int64_t lda, const float *B, int64_t ldb,
                                  float beta, float *C, int64_t ldc) {
  return gemm_dev<float>(d, transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc);
}

extern "C" wg_status wg_dgemm_dev(wg_device *d, int transA, int transB, int64_t m, int64_t n, int64_t k,
                                  double alpha, const double *A, int64_t lda, const double *B,
                                  int64_t ldb, double beta, double *C, int64_t ldc) {
  return gemm_dev<double>(d, transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc);
}

extern "C" wg_status wg_sgemm_host(wg_device *d, int transA, int transB, int64_t m, int64_t n, int64_t k,
                                   float alpha, const float *A, int64_t lda, const float *B, int64_t ldb,
                                   float beta, const float *C_in, float *C_out, int64_t ldc,
                                   float *gpu_ms) {
  return gemm_host<float>(d, transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C_in, C_out, ldc, gpu_ms);
}

extern "C" wg_status wg_dgemm_host(wg_device *d, int transA, int transB, int64_t m, int64_t n, int64_t k,
                                   double alpha, const double *A, int64_t lda, const double *B,
                                   int64_t ldb, double beta, const double *C_in, double *C_out,
                                   int64_t ldc, float *gpu_ms) {
  return gemm_host<double>(d, transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C_in, C_out, ldc,
                           gpu_ms);
}

// ---- the gemmtr family (src/sgemmtr/sgemmtr.mjs, src/dgemmtr/dgemmtr.mjs) ----
// sgemm/dgemm with only the `uplo` triangle of C read or written; ssyrk/ssyr2k
// and the d variants are built on these, as the reference builds them on its
// gemmtr kernel (src/ssyrk/ssyrk.mjs:31, src/ssyr2k/ssyr2k.mjs:25-26).

extern "C" wg_status wg_sgemmtr(wg_device *d, int uplo, int transA, int transB, int64_t m, int64_t n, int64_t k,
                                float alpha, const wg_buffer *A, int64_t offA, int64_t lda, const wg_buffer *B,
                                int64_t offB, int64_t ldb, float beta, wg_buffer *C, int64_t offC, int64_t ldc,
                                float *gpu_ms) {
  if (uplo != WG_UPLO_LOWER && uplo != WG_UPLO_UPPER)
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "uplo must be 'lower' or 'upper'.");
  return gemm_buffers<float>(d, transA, transB, m, n, k, alpha, A, offA, lda, B, offB, ldb, beta, C, offC, ldc,
                             gpu_ms, uplo);
}

extern "C" wg_status wg_dgemmtr(wg_device *d, int uplo, int transA, int transB, int64_t m, int64_t n, int64_t k,
                                double alpha, const wg_buffer *A, int64_t offA, int64_t lda, const wg_buffer *B,
                                int64_t offB, int64_t ldb, double beta, wg_buffer *C, int64_t offC, int64_t ldc,
                                float *gpu_ms) {
  if (uplo != WG_UPLO_LOWER && uplo != WG_UPLO_UPPER)
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "uplo must be 'lower' or 'upper'.");
  return gemm_buffers<double>(d, transA, transB, m, n, k, alpha, A, offA, lda, B, offB, ldb, beta, C, offC, ldc,
                              gpu_ms, uplo);
}

extern "C" wg_status wg_sgemmtr_dev(wg_device *d, int uplo, int transA, int transB, int64_t m, int64_t n,
                                    int64_t k, float alpha, const float *A, int64_t lda, const float *B,
                                    int64_t ldb, float beta, float *C, int64_t ldc) {
  if (uplo != WG_UPLO_LOWER && uplo != WG_UPLO_UPPER)
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "uplo must be 'lower' or 'upper'.");
  return gemm_dev<float>(d, transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, uplo);
}

extern "C" wg_status wg_dgemmtr_dev(wg_device *d, int uplo, int transA, int transB, int64_t m, int64_t n,
                                    int64_t k, double alpha, const double *A, int64_t lda, const double *B,
                                    int64_t ldb, double beta, double *C, int64_t ldc) {
  if (uplo != WG_UPLO_LOWER && uplo != WG_UPLO_UPPER)
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "uplo must be 'lower' or 'upper'.");
  return gemm_dev<double>(d, transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, uplo);
}

extern "C" wg_status wg_sgemmtr_host(wg_device *d, int uplo, int transA, int transB, int64_t m, int64_t n,
                                     int64_t k, float alpha, const float *A, int64_t lda, const float *B,
                                     int64_t ldb, float beta, const float *C_in, float *C_out, int64_t ldc,
                                     float *gpu_ms) {
  if (uplo != WG_UPLO_LOWER && uplo != WG_UPLO_UPPER)
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "uplo must be 'lower' or 'upper'.");
  return gemm_host<float>(d, transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C_in, C_out, ldc, gpu_ms,
                          uplo);
}

extern "C" wg_status wg_dgemmtr_host(wg_device *d, int uplo, int transA, int transB, int64_t m, int64_t n,
                                     int64_t k, double alpha, const double *A, int64_t lda, const double *B,
                                     int64_t ldb, double beta, const double *C_in, double *C_out, int64_t ldc,
                                     float *gpu_ms) {
  if (uplo != WG_UPLO_LOWER && uplo != WG_UPLO_UPPER)
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "uplo must be 'lower' or 'upper'.");
  return gemm_host<double>(d, transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C_in, C_out, ldc, gpu_ms,
                           uplo);
}
