// Internal declarations shared by the wgblas-b200 translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <vector>

#include "../../include/wgblas.h"

// Device-side status words, one small array per device handle.
enum {
  WG_DW_ERROR = 0,     // bitmask of WG_DERR_* set by kernels whose bounded waits gave up
  WG_DW_FALLBACK = 1,  // epoch of the latest sgemm call whose operands ruled out 3xTF32
  WG_DW_FALLBACKS = 2, // number of FFMA fallbacks run because of WG_DW_FALLBACK
  WG_DW_COUNT = 8
};
// Bits of WG_DW_ERROR.
enum {
  WG_DERR_TMA_WAIT = 1u,  // producer or consumer gave up waiting on a pipeline stage
  WG_DERR_MMA_WAIT = 2u,  // the epilogue gave up waiting for the accumulator
  WG_DERR_TMEM = 4u       // TMEM allocation returned an unusable address
};

struct wg_device {
  int ordinal;
  unsigned flags;
  cudaStream_t own_stream;
  cudaStream_t stream;  // the stream work is ordered on (own_stream or the caller's)
  cudaEvent_t ev_start, ev_stop;
  int sm_count;
  int tc_grid_cap;  // > 0: at most this many CTAs in the 3xTF32 persistent grid
  int cc_major, cc_minor;
  size_t total_mem;
  char name[256];
  void *ws;          // grow-only scratch for the 3xTF32 operand split
  size_t ws_bytes;
  unsigned *dwords;  // WG_DW_COUNT device words
  uint32_t epoch;    // sgemm call counter, tags WG_DW_FALLBACK
  int sgemm_path;
  int dgemm_path;
  cudaStream_t h2d, d2h;  // copy streams of the host-array path (created on first use)
  cudaMemPool_t staging;  // device copies of host-array operands; keeps its memory between calls
  wg_sgemm_stats stats;
  uint64_t launches;  // kernels launched on this handle
  // profiling: event pairs waiting to be summed, and per-family totals
  bool profiling;
  struct pending_t { int family; cudaEvent_t e0, e1; };
  std::vector<pending_t> pending;
  std::vector<cudaEvent_t> event_pool;
  std::vector<std::string> families;
  std::vector<uint64_t> fam_launches;
  std::vector<double> fam_ms;
};

// Brackets one kernel launch for per-kernel profiling and counts it.
struct wg_launch_scope {
  wg_device *d;
  int slot;
  wg_launch_scope(wg_device *dev, const char *family);
  ~wg_launch_scope();
};

struct wg_buffer {
  wg_device *dev;
  void *ptr;
  size_t bytes;
};

// Records a message for wg_last_error() on this thread and returns `st`.
wg_status wg_fail(wg_status st, const char *fmt, ...);

#define WG_CUDA(call)                                                                   \
  do {                                                                                  \
    cudaError_t e_ = (call);                                                            \
    if (e_ != cudaSuccess)                                                              \
      return wg_fail(e_ == cudaErrorMemoryAllocation ? WG_ERR_OUT_OF_MEMORY : WG_ERR_CUDA, \
                     "%s failed: %s", #call, cudaGetErrorString(e_));                   \
  } while (0)

// Makes `ordinal` current for the lifetime of the guard.
struct wg_device_guard {
  int prev;
  bool changed;
  explicit wg_device_guard(int ordinal) : prev(-1), changed(false) {
    if (cudaGetDevice(&prev) == cudaSuccess && prev != ordinal) {
      cudaSetDevice(ordinal);
      changed = true;
    }
  }
  ~wg_device_guard() {
    if (changed) cudaSetDevice(prev);
  }
};

// Queues C = alpha*op(A)op(B) + beta*C on d->stream through the kernel
// dispatcher (no argument checks, no dgemm quick return: callers check).
template <typename T>
wg_status wg_gemm_enqueue(wg_device *d, int transA, int transB, int64_t m, int64_t n, int64_t k, T alpha,
                          const T *A, int64_t lda, const T *B, int64_t ldb, T beta, T *C, int64_t ldc);

// One column panel (cols columns) of a product queued panel by panel on
// d->stream. sgemm panels on the 3xTF32 path split op(A) only for the first
// panel (first = true), share `epoch` (wg_next_epoch) across the product, and
// keep their split operands in one workspace of ws_bytes
// (wg_tf32x3_panels_workspace over all the product's panel widths) so op(A)'s
// split stays in place; other calls go through the dispatcher.
template <typename T>
wg_status wg_gemm_panel(wg_device *d, bool first, uint32_t epoch, int transA, int transB, int64_t m, int64_t cols,
                        int64_t k, T alpha, const T *A, int64_t lda, const T *B, int64_t ldb, T beta, T *C, int64_t ldc,
                        size_t ws_bytes);
template <>
wg_status wg_gemm_panel<float>(wg_device *d, bool first, uint32_t epoch, int transA, int transB, int64_t m,
                               int64_t cols, int64_t k, float alpha, const float *A, int64_t lda, const float *B,
                               int64_t ldb, float beta, float *C, int64_t ldc, size_t ws_bytes);
// True when wg_gemm_panel<float> runs this panel shape on the 3xTF32 kernel.
bool wg_sgemm_panel_on_tc(const wg_device *d, float alpha, int64_t m, int64_t cols, int64_t k);
// Scratch for every panel of an m x (sum of widths) x k sgemm on the 3xTF32 path.
size_t wg_tf32x3_panels_workspace(const wg_device *d, int64_t m, int64_t k, const int64_t *widths, size_t count);

// Returns at least `bytes` of device scratch owned by the handle (stream-ordered reuse).
wg_status wg_workspace(wg_device *dev, size_t bytes, void **ptr);

// ---- kernel launchers (gemm_simt.cu, sgemm_tf32x3.cu) ----

// C = alpha*op(A)op(B) + beta*C on the FFMA / DFMA pipes, sequential k per element.
// When only_if_epoch != 0 every CTA first reads dwords[WG_DW_FALLBACK] and exits
// unless it equals only_if_epoch (the device-side fallback of the 3xTF32 path).
template <typename T>
cudaError_t wg_launch_gemm_simt(cudaStream_t s, int transA, int transB, int64_t m, int64_t n,
                                int64_t k, T alpha, const T *A, int64_t lda, const T *B,
                                int64_t ldb, T beta, T *C, int64_t ldc, unsigned *dwords,
                                uint32_t only_if_epoch);

// dgemm on the FP64 tensor-core (DMMA) path, mma.sync.m16n8k8.f64 (dgemm_dmma.cu).
cudaError_t wg_launch_dgemm_dmma(cudaStream_t s, int transA, int transB, int64_t m, int64_t n, int64_t k,
                                 double alpha, const double *A, int64_t lda, const double *B, int64_t ldb,
                                 double beta, double *C, int64_t ldc);

// C = (alpha == 0 ? 0 : alpha*0) + beta*C elementwise — the k == 0 / alpha == 0 cases.
template <typename T>
cudaError_t wg_launch_scale(cudaStream_t s, int64_t m, int64_t n, T alpha, T beta, T *C,
                            int64_t ldc);

// Bytes of scratch the 3xTF32 path needs for this shape: the split operands
// alone (whole-tile scheduling), or with the stream-K partial sums and counters.
size_t wg_tf32x3_workspace_bytes(int64_t m, int64_t n, int64_t k);
size_t wg_tf32x3_workspace_bytes_sk(const wg_device *dev, int64_t m, int64_t n, int64_t k);
// SMs the 3xTF32 kernel's persistent grid may use on this handle (all of them
// unless tc_grid_cap holds some back, e.g. for NCCL kernels running alongside).
int wg_tf32x3_sms(const wg_device *dev);
// Modelled run time of the 3xTF32 kernel for one m x n x k product on G SMs, in
// units of one 16-deep k-block of one tile's MMAs (about 0.5 us on B200).
double wg_tf32x3_cost(int G, int64_t m, int64_t n, int64_t k);
// True when the 3xTF32 path supports this shape on this device.
bool wg_tf32x3_supported(const wg_device *dev, int64_t m, int64_t n, int64_t k);
// Splits op(A), op(B) into tf32 hi/lo operands in `ws`, then runs the tcgen05 kernel.
// Operands outside the split's exact range make the kernel exit and the FFMA
// kernel (launched right after, gated on the same epoch) compute C instead.
// `ws` holds ws_bytes: stream-K scheduling is used when it also fits the
// partial sums (wg_tf32x3_workspace_bytes_sk), whole tiles otherwise.
wg_status wg_sgemm_tf32x3(wg_device *dev, int transA, int transB, int64_t m, int64_t n,
                          int64_t k, float alpha, const float *A, int64_t lda, const float *B,
                          int64_t ldb, float beta, float *C, int64_t ldc, void *ws, size_t ws_bytes);
// The same, for one column panel of a larger product: pack_a = false reuses the
// op(A) split left in `ws` by an earlier panel of the same m x k operand, and all
// panels of one product share `epoch` (wg_next_epoch) so a flagged operand sends
// that panel and every later one to the FFMA kernel.
wg_status wg_sgemm_tf32x3_panel(wg_device *dev, int transA, int transB, int64_t m, int64_t n, int64_t k,
                                float alpha, const float *A, int64_t lda, const float *B, int64_t ldb, float beta,
                                float *C, int64_t ldc, void *ws, size_t ws_bytes, bool pack_a, uint32_t epoch);
uint32_t wg_next_epoch(wg_device *dev);
