/*
 * wgblas-b200 C ABI — the drop-in boundary under wgblas's JavaScript API for
 * the level-3 GEMM path (sgemm / dgemm), built for B200 (sm_100a).
 *
 * Every function returns a wg_status; on failure wg_last_error() gives the
 * message (per calling thread). No torch or CUDA types appear in signatures:
 * streams are passed as void*.
 *
 * GEMM calls use the column-major BLAS frame (Fortran BLAS convention):
 *   C[i + j*ldc] := alpha * sum_p op(A)(i,p) * op(B)(p,j) + beta * C[i + j*ldc]
 *   op(A)(i,p) = transA ? A[p + i*lda] : A[i + p*lda]        (i < m, p < k)
 *   op(B)(p,j) = transB ? B[j + p*ldb] : B[p + j*ldb]        (p < k, j < n)
 * The language layer maps wgblas's row-major default and per-matrix layouts
 * onto this frame, as src/sgemm/sgemm.mjs:151-167 maps them onto its row-major
 * kernel frame.
 *
 * BLAS rules kept from the reference:
 *   - m == 0 or n == 0 returns without touching C (src/sgemm/sgemm.mjs:83);
 *   - alpha == 0 reads neither A nor B, so NaN/Inf there cannot reach C
 *     (src/shaders/sgemm_large.wgsl:299-303);
 *   - beta == 0 does not read C, so NaN/Inf already in C are overwritten
 *     (sgemm_large.wgsl:296-298);
 *   - sgemm with k == 0 still writes alpha*0 + beta*C (tests/sgemm/src/test.sgemm.js:304-351);
 *   - dgemm returns C untouched when (alpha == 0 or k == 0) and beta == 1
 *     (src/dgemm/dgemm.mjs:177-179);
 *   - elements of C outside the m x n block (leading-dimension padding) are
 *     never written.
 */
#ifndef WGBLAS_H
#define WGBLAS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define WG_ABI_VERSION 1

typedef enum wg_status {
  WG_OK = 0,
  WG_ERR_INVALID_ARGUMENT = 1, /* a size, stride, pointer or flag is out of range */
  WG_ERR_OUT_OF_MEMORY = 2,    /* device or pinned host allocation failed */
  WG_ERR_CUDA = 3,             /* a CUDA runtime or driver call failed */
  WG_ERR_NO_DEVICE = 4,        /* no CUDA device, or the ordinal does not exist */
  WG_ERR_KERNEL_TIMEOUT = 5,   /* a bounded device-side wait gave up (see wg_device_check) */
  WG_ERR_NCCL = 6,             /* a collective failed or timed out */
  WG_ERR_NOT_SUPPORTED = 7     /* the device is not sm_100 or the feature is absent */
} wg_status;

typedef struct wg_device wg_device;
typedef struct wg_buffer wg_buffer;

/* Message of the last failing call on this thread ("" if none). */
const char *wg_last_error(void);
/* WG_ABI_VERSION of the loaded library. */
int wg_abi_version(void);

/* ---- devices: replace src/init.mjs:31-143 (init / cleanup / gpuName) ------ */

/* Number of visible CUDA devices (0 when none). */
wg_status wg_device_count(int *count);

#define WG_DEVICE_TIMING 1u /* benchmark mode: GEMM calls can report gpu_ms */

/* Opens a handle on CUDA device `ordinal` with its own non-blocking stream.
 * Several handles may name the same ordinal (src/init.mjs:14-29 creates one
 * device per option set); each has its own stream. */
wg_status wg_device_open(int ordinal, unsigned flags, wg_device **out);
/* Waits for the handle's work, then releases its stream and workspace
 * (src/init.mjs:110-131). Buffers allocated on it must be freed first or are
 * leaked. */
wg_status wg_device_close(wg_device *dev);
/* Device name, as gpuName() reports it (src/init.mjs:133-143). */
wg_status wg_device_name(const wg_device *dev, char *buf, size_t len);
typedef struct wg_device_props {
  int ordinal;
  int sm_count;
  int cc_major, cc_minor;
  size_t total_mem;
  unsigned flags;
} wg_device_props;
wg_status wg_device_props_get(const wg_device *dev, wg_device_props *props);
/* The stream all of this handle's work is ordered on (a cudaStream_t). */
wg_status wg_device_stream(const wg_device *dev, void **stream);
/* Orders this handle's work on a caller-owned cudaStream_t instead; NULL
 * restores the handle's own stream. */
wg_status wg_device_set_stream(wg_device *dev, void *stream);
/* Waits until the handle's stream is idle. */
wg_status wg_device_sync(wg_device *dev);
/* Waits, then reports (and clears) a device-side error word: WG_ERR_KERNEL_TIMEOUT
 * when a kernel's bounded wait gave up since the last check. */
wg_status wg_device_check(wg_device *dev);
/* Failure-detection self-test (no counterpart in the reference). Queues one
 * CTA that waits, with the same clock-bounded mbarrier wait the tensor-core
 * kernels use, on a barrier nothing completes: after about budget_us
 * microseconds (at most 1 s) of SM clock the wait gives up, the kernel records
 * the timeout in the device error word and returns. The next wg_device_check
 * reports WG_ERR_KERNEL_TIMEOUT (and clears the word); the context stays usable. */
wg_status wg_selftest_bounded_wait(wg_device *dev, unsigned budget_us);


/* Counters of the sgemm dispatcher since the handle was opened (synchronises). */
typedef struct wg_sgemm_stats {
  uint64_t calls;           /* sgemm calls that reached a kernel */
  uint64_t tf32x3_launches; /* calls dispatched to the 3xTF32 tensor-core kernel */
  uint64_t simt_launches;   /* calls dispatched straight to an FFMA kernel (either tile size) */
  uint64_t fallbacks;       /* 3xTF32 calls that found non-finite or out-of-range
                               operands on the device and computed C (or the affected
                               tiles) on the FFMA pipe instead, with the FFMA kernel's bits */
} wg_sgemm_stats;
wg_status wg_device_sgemm_stats(wg_device *dev, wg_sgemm_stats *stats);

/* How the 3xTF32 tensor-core kernel would divide an m x n x k product among
 * sm_count SMs: 128 x 256 output tiles, each k_blocks 16-wide k steps; a
 * persistent grid of `grid` CTAs takes whole_tiles tiles whole and cuts the
 * remaining split_tiles into split_segments k-segments each (1 = none). Host
 * arithmetic only: no device is touched. workspace_bytes is the scratch that
 * plan needs (split operands and partial sums). No counterpart in the
 * reference; it documents the scheduling for tests and tuning. */
typedef struct wg_tc_plan {
  int64_t tiles_m, tiles_n, k_blocks;
  int grid, whole_tiles, split_tiles, split_segments;
  size_t workspace_bytes;
} wg_tc_plan;
wg_status wg_sgemm_tc_plan(int sm_count, int64_t m, int64_t n, int64_t k, wg_tc_plan *out);

/* Triangle selector of the gemmtr family (sgemmtr/ssyrk/ssyr2k and the d
 * variants): only that triangle of C is read or written. In the column-major
 * frame of this API: LOWER is C(i, j) with j <= i, UPPER j >= i (C need not be
 * square). FULL is plain GEMM. */
#define WG_UPLO_FULL 0
#define WG_UPLO_LOWER 1
#define WG_UPLO_UPPER 2

/* sgemm kernel choice: AUTO picks by shape and alignment; the others force one
 * kernel (tests and benchmarks). TF32X3 is the tensor-core path (the fused
 * kernel that splits its own operands where the operands' alignment allows its
 * tensor maps, else the split pass + MMA kernel); TF32X3_PACKED forces the
 * split pass + MMA kernel; TF32X3_FUSED_BN256/128/64 force the fused kernel
 * with one tile width and TF32X3_PAIR its CTA-pair form (they must be
 * supported for the call). */
#define WG_SGEMM_AUTO 0
#define WG_SGEMM_SIMT 1
#define WG_SGEMM_TF32X3 2
#define WG_SGEMM_TF32X3_PACKED 3
#define WG_SGEMM_TF32X3_FUSED_BN256 4
#define WG_SGEMM_TF32X3_FUSED_BN128 5
#define WG_SGEMM_TF32X3_FUSED_BN64 6
#define WG_SGEMM_TF32X3_PAIR 7  /* the fused kernel over CTA pairs (256 x 256 tiles) */
#define WG_SGEMM_SIMT_SMALL 8  /* the FFMA arithmetic of SIMT on 32 x 64 tiles (small products) */
wg_status wg_device_set_sgemm_path(wg_device *dev, int path);
/* dgemm kernel choice: AUTO picks by shape; SIMT forces the DFMA kernel (one
 * sequential FMA chain per element), DMMA the FP64 tensor-core kernel. */
#define WG_DGEMM_AUTO 0
#define WG_DGEMM_SIMT 1
#define WG_DGEMM_DMMA 2
wg_status wg_device_set_dgemm_path(wg_device *dev, int path);
/* strsm algorithm: AUTO picks by shape; RECURSIVE halves the triangle and runs
 * the off-diagonal updates as GEMMs (one launch per update and per 64-row
 * diagonal block); FLOW runs the whole solve in one cooperative launch per
 * group of 64-column right-hand-side chunks: each CTA owns 64-row blocks,
 * updates them as earlier blocks are published and solves them in turn. */
#define WG_STRSM_AUTO 0
#define WG_STRSM_RECURSIVE 1
#define WG_STRSM_FLOW 2
wg_status wg_device_set_strsm_path(wg_device *dev, int path);

/* Per-kernel device time of this handle's own launches, for benchmarks and
 * roofline reports. While profiling is on, every kernel the library launches
 * on the handle is bracketed by CUDA events on its stream. */
wg_status wg_device_set_profiling(wg_device *dev, int on);
typedef struct wg_kernel_profile {
  char name[48];     /* kernel family, e.g. "sgemm_simt", "sgemm_tf32x3_mma" */
  uint64_t launches; /* launches since the last read */
  double total_ms;   /* summed device time of those launches */
} wg_kernel_profile;
/* Waits for the handle's work, fills up to `max` entries, sets *count, and
 * resets the accumulators. */
wg_status wg_device_profile_read(wg_device *dev, wg_kernel_profile *out, int max, int *count);
/* Kernels the library has launched on this handle since it was opened. */
wg_status wg_device_kernel_launches(const wg_device *dev, uint64_t *launches);

/* ---- roofline probes: benchmarks/roofline (FMA peak and bandwidth) ------- */
#define WG_PROBE_FP32_FMA 0 /* value: TFLOP/s of FFMA chains on every SM */
#define WG_PROBE_FP64_FMA 1 /* value: TFLOP/s of DFMA chains on every SM */
#define WG_PROBE_HBM_COPY 2 /* value: GB/s (read + write) of a 2 GiB device copy */
#define WG_PROBE_FP64_DMMA 3 /* value: TFLOP/s of FP64 tensor-core (mma.sync f64) chains */
#define WG_PROBE_HBM_READ 4 /* value: GB/s of a 2 GiB read-only pass */
#define WG_PROBE_HBM_SCALE 5 /* value: GB/s (read + write) of a 2 GiB in-place scale */
wg_status wg_probe_peak(wg_device *dev, int kind, double *value);

/* ---- device buffers: replace the storage of GpuMatrix / GpuVector ------- */
/* (src/classes/GpuMatrix.mjs:43-207, src/util/buffer.mjs:58-78,134-227)     */

wg_status wg_buffer_alloc(wg_device *dev, size_t bytes, wg_buffer **out);
/* A temporary for work queued on the device stream: its memory comes from the
 * handle's stream-ordered pool (no mapping once the pool has grown to the
 * size), valid for work queued on that stream after this call. Not for host
 * copies (wg_buffer_upload / download). wg_buffer_free returns it to the pool in
 * stream order, without waiting; free it before wg_device_close. */
wg_status wg_buffer_alloc_async(wg_device *dev, size_t bytes, wg_buffer **out);
/* Frees a buffer: wg_buffer_alloc's after the work queued on the device stream
 * has finished (it waits), wg_buffer_alloc_async's in stream order. */
wg_status wg_buffer_free(wg_buffer *buf);
wg_status wg_buffer_size(const wg_buffer *buf, size_t *bytes);
wg_status wg_buffer_device_ptr(const wg_buffer *buf, void **ptr);
/* Copies `bytes` from host memory into the buffer at byte `offset`, ordered on
 * the device stream; returns once the host memory may be reused. */
wg_status wg_buffer_upload(wg_buffer *buf, size_t offset, const void *host, size_t bytes);
/* Copies from the buffer to host memory; returns when the data has arrived. */
wg_status wg_buffer_download(const wg_buffer *buf, size_t offset, void *host, size_t bytes);
/* Strided forms: `rows` chunks of `width` bytes, `spitch`/`dpitch` bytes apart
 * (GpuMatrix.read() strips lda padding this way, src/classes/GpuMatrix.mjs:193-201). */
wg_status wg_buffer_upload_2d(wg_buffer *buf, size_t offset, size_t dpitch, const void *host,
                              size_t spitch, size_t width, size_t rows);
wg_status wg_buffer_download_2d(const wg_buffer *buf, size_t offset, size_t spitch, void *host,
                                size_t dpitch, size_t width, size_t rows);

/* Page-locked host memory: copies from/to it run at full PCIe rate and
 * asynchronously. */
wg_status wg_host_alloc(size_t bytes, void **ptr);
wg_status wg_host_free(void *ptr);

/* ---- GEMM on device buffers: replace src/sgemm/sgemm.mjs:25-269 and ----- */
/* ---- src/dgemm/dgemm.mjs:23-318 with their WGSL kernels -------------------- */
/* off* are element offsets into the buffers. gpu_ms, when non-NULL on a
 * handle opened with WG_DEVICE_TIMING, receives the kernel time measured with
 * CUDA events (the reference's gpuTimeMs, src/util/benchmark.mjs:93-103); the
 * call then waits for completion. Otherwise the call returns once the work is
 * queued on the device stream. */
wg_status wg_sgemm(wg_device *dev, int transA, int transB, int64_t m, int64_t n, int64_t k,
                   float alpha, const wg_buffer *A, int64_t offA, int64_t lda,
                   const wg_buffer *B, int64_t offB, int64_t ldb, float beta,
                   wg_buffer *C, int64_t offC, int64_t ldc, float *gpu_ms);
wg_status wg_dgemm(wg_device *dev, int transA, int transB, int64_t m, int64_t n, int64_t k,
                   double alpha, const wg_buffer *A, int64_t offA, int64_t lda,
                   const wg_buffer *B, int64_t offB, int64_t ldb, double beta,
                   wg_buffer *C, int64_t offC, int64_t ldc, float *gpu_ms);

/* GEMM on raw device pointers already on this handle's device, ordered on its
 * stream (interop with other CUDA code). Same semantics as wg_sgemm. */
wg_status wg_sgemm_dev(wg_device *dev, int transA, int transB, int64_t m, int64_t n, int64_t k,
                       float alpha, const float *A, int64_t lda, const float *B, int64_t ldb,
                       float beta, float *C, int64_t ldc);
wg_status wg_dgemm_dev(wg_device *dev, int transA, int transB, int64_t m, int64_t n, int64_t k,
                       double alpha, const double *A, int64_t lda, const double *B, int64_t ldb,
                       double beta, double *C, int64_t ldc);

/* sgemm that allocates nothing — no counterpart in the reference. For callers
 * that must not have the library call cudaMalloc for them (an application whose
 * own allocator owns all device memory, a real-time loop that cannot stall on an
 * allocation). It runs the 3xTF32 tensor-core kernels with their split-operand
 * scratch in a fixed WG_NOALLOC_SCRATCH_BYTES array inside the library (held by
 * every GPU that loads the library until exit); A, B and C are device pointers
 * on this handle's device, ordered on its stream. It needs k >= 8 (alpha == 0 or
 * k == 0 only scale C) and rejects, with WG_ERR_INVALID_ARGUMENT, shapes whose
 * scratch 2*(round_up(m,128) + round_up(n,256))*round_up(k,32)*4 bytes exceeds
 * the array. The array is reserved on a GPU when a handle to it is opened
 * (wg_device_open looks up its address, so CUDA's lazy module loading cannot
 * defer the reservation to the first call): open the handle before your own
 * allocator takes the device's memory. All calls on a device share the array:
 * calls that overlap on the GPU race, so order them on one stream. */
#define WG_NOALLOC_SCRATCH_BYTES ((size_t)64 << 20)
wg_status wg_sgemm_noalloc(wg_device *dev, int transA, int transB, int64_t m, int64_t n, int64_t k,
                           float alpha, const float *A, int64_t lda, const float *B, int64_t ldb,
                           float beta, float *C, int64_t ldc);

/* GEMM on host arrays — the typed-array path of sgemm()/dgemm()
 * (src/sgemm/sgemm.mjs:179-262): uploads op(A), op(B) and (when beta != 0) the
 * m x n block of C, runs the kernel, and writes the m x n block of the result
 * into C_out (which may be C_in; its other elements are not touched). Returns
 * when C_out holds the result. Page-locked host arrays (wg_host_alloc) are
 * copied asynchronously at full rate. */
wg_status wg_sgemm_host(wg_device *dev, int transA, int transB, int64_t m, int64_t n, int64_t k,
                        float alpha, const float *A, int64_t lda, const float *B, int64_t ldb,
                        float beta, const float *C_in, float *C_out, int64_t ldc, float *gpu_ms);
wg_status wg_dgemm_host(wg_device *dev, int transA, int transB, int64_t m, int64_t n, int64_t k,
                        double alpha, const double *A, int64_t lda, const double *B, int64_t ldb,
                        double beta, const double *C_in, double *C_out, int64_t ldc,
                        float *gpu_ms);

/* Column-panel widths wg_sgemm_sharded uses when panel_cols is 0 and the
 * product runs on the 3xTF32 kernel (alpha != 0, k >= 64, transB = 0): panels
 * sized so each GEMM fills whole waves of the SMs and the first panel's
 * broadcast is short. Host arithmetic only; sm_count is the SMs of one GPU.
 * `count` receives the number of panels even when `capacity` is too small. */
wg_status wg_sharded_panel_plan(int sm_count, int nranks, int64_t m_local, int64_t n, int64_t k, int64_t *widths,
                                size_t capacity, size_t *count);


/* ---- the gemmtr family ------------------------------------------------------
 * sgemm / dgemm restricted to one triangle of C: C := uplo(alpha*op(A)*op(B) +
 * beta*C), only the WG_UPLO_LOWER or WG_UPLO_UPPER triangle (column-major frame)
 * read or written, tiles wholly outside it skipped. Replaces sgemmtr/dgemmtr
 * (src/sgemmtr/sgemmtr.mjs:25-278, src/dgemmtr/dgemmtr.mjs); the reference's
 * ssyrk/ssyr2k/dsyrk/dsyr2k are compositions of these (B := A; two passes, the
 * second with beta = 1) and are composed the same way by the language layer.
 * dgemmtr keeps dgemm's quick return ((alpha == 0 or k == 0) and beta == 1). */
wg_status wg_sgemmtr(wg_device *dev, int uplo, int transA, int transB, int64_t m, int64_t n, int64_t k, float alpha,
                     const wg_buffer *A, int64_t offA, int64_t lda, const wg_buffer *B, int64_t offB, int64_t ldb,
                     float beta, wg_buffer *C, int64_t offC, int64_t ldc, float *gpu_ms);
wg_status wg_dgemmtr(wg_device *dev, int uplo, int transA, int transB, int64_t m, int64_t n, int64_t k,
                     double alpha, const wg_buffer *A, int64_t offA, int64_t lda, const wg_buffer *B, int64_t offB,
                     int64_t ldb, double beta, wg_buffer *C, int64_t offC, int64_t ldc, float *gpu_ms);
wg_status wg_sgemmtr_dev(wg_device *dev, int uplo, int transA, int transB, int64_t m, int64_t n, int64_t k,
                         float alpha, const float *A, int64_t lda, const float *B, int64_t ldb, float beta,
                         float *C, int64_t ldc);
wg_status wg_dgemmtr_dev(wg_device *dev, int uplo, int transA, int transB, int64_t m, int64_t n, int64_t k,
                         double alpha, const double *A, int64_t lda, const double *B, int64_t ldb, double beta,
                         double *C, int64_t ldc);
/* Host arrays; C_out receives C_in with the triangle updated. */
wg_status wg_sgemmtr_host(wg_device *dev, int uplo, int transA, int transB, int64_t m, int64_t n, int64_t k,
                          float alpha, const float *A, int64_t lda, const float *B, int64_t ldb, float beta,
                          const float *C_in, float *C_out, int64_t ldc, float *gpu_ms);
wg_status wg_dgemmtr_host(wg_device *dev, int uplo, int transA, int transB, int64_t m, int64_t n, int64_t k,
                          double alpha, const double *A, int64_t lda, const double *B, int64_t ldb, double beta,
                          const double *C_in, double *C_out, int64_t ldc, float *gpu_ms);

/* ---- operand passes of ssymm/dsymm and strmm/dtrmm -------------------------
 * The reference runs these routines as a pass that materializes a dense copy of
 * the symmetric / triangular operand followed by a plain GEMM
 * (src/ssymm/ssymm.mjs:26-28, src/strmm/strmm.mjs); the language layer does the
 * same with these passes and the GEMM entry points. Column-major frame; n x n
 * matrices of elem_bytes (4: f32, 8: f64) at element offsets and leading
 * dimensions; `uplo` names the stored triangle (WG_UPLO_LOWER: i >= j). */
/* out := the symmetric matrix whose `uplo` triangle A holds. */
wg_status wg_symmetrize(wg_device *dev, int elem_bytes, int uplo, int64_t n, const wg_buffer *A, int64_t offA,
                        int64_t lda, wg_buffer *out, int64_t offO, int64_t ldo);
/* out := T or T^T (trans), where T is A's `uplo` triangle with zeros elsewhere and,
 * when unit = 1, ones on the diagonal (A's diagonal not read). */
wg_status wg_triangularize(wg_device *dev, int elem_bytes, int uplo, int trans, int unit, int64_t n,
                           const wg_buffer *A, int64_t offA, int64_t lda, wg_buffer *out, int64_t offO, int64_t ldo);
/* Copies `rows` rows of `width` bytes between device buffers (byte offsets and
 * pitches), queued on the device stream. */
wg_status wg_buffer_copy_2d(wg_device *dev, const wg_buffer *src, size_t src_off, size_t src_pitch, wg_buffer *dst,
                            size_t dst_off, size_t dst_pitch, size_t width, size_t rows);

/* ---- strsm (src/strsm/strsm.mjs:160-583) -----------------------------------
 * B := alpha * op(A)^-1 * B (side WG_SIDE_LEFT) or alpha * B * op(A)^-1
 * (WG_SIDE_RIGHT) in place, in the column-major frame: B is m x n with ldb >= m,
 * A is the order x order triangle (order = m for left, n for right) whose `uplo`
 * triangle (WG_UPLO_LOWER / WG_UPLO_UPPER) is read; the other triangle is never
 * read, nor the diagonal when diag is WG_DIAG_UNIT. transA: 0 = op(A) = A,
 * 1 = A^T. alpha = 0 writes zeros to B without reading A or B. m or n = 0
 * returns at once. Queued on the device stream; gpu_ms as for wg_sgemm. A
 * singular A gives Infinity / NaN as substitution does, no error. */
#define WG_SIDE_LEFT 0
#define WG_SIDE_RIGHT 1
#define WG_DIAG_NON_UNIT 0
#define WG_DIAG_UNIT 1
wg_status wg_strsm(wg_device *dev, int side, int uplo, int transA, int diag, int64_t m, int64_t n, float alpha,
                   const wg_buffer *A, int64_t offA, int64_t lda, wg_buffer *B, int64_t offB, int64_t ldb,
                   float *gpu_ms);
/* The same on raw device pointers of the device (no size checks). */
wg_status wg_strsm_dev(wg_device *dev, int side, int uplo, int transA, int diag, int64_t m, int64_t n, float alpha,
                       const float *A, int64_t lda, float *B, int64_t ldb);

/* ---- sgemv / dgemv (src/sgemv/sgemv.mjs, src/dgemv/dgemv.mjs) -------------
 * y := alpha * op(A) * x + beta * y in the column-major frame: A is m x n with
 * lda >= m; trans 0: op(A) = A, x has n entries, y has m; trans 1: op(A) = A^T,
 * x has m entries, y has n. incx, incy > 0 (element strides); offsets in
 * elements. m or n = 0, and alpha = 0 with beta = 1, return without touching
 * y. alpha = 0 scales y by beta without reading A or x (zeros when beta = 0);
 * beta = 0 does not read y. For trans 0 a column whose x entry is +-0 adds
 * exactly 0 (reference BLAS skips it), so Infinity or NaN in that column of A
 * does not reach y. dgemv computes in native fp64 (the reference emulates
 * fp64 with f32 pairs). Queued on the device stream; gpu_ms as for wg_sgemm. */
wg_status wg_sgemv(wg_device *dev, int trans, int64_t m, int64_t n, float alpha, const wg_buffer *A, int64_t offA,
                   int64_t lda, const wg_buffer *x, int64_t offx, int64_t incx, float beta, wg_buffer *y,
                   int64_t offy, int64_t incy, float *gpu_ms);
wg_status wg_dgemv(wg_device *dev, int trans, int64_t m, int64_t n, double alpha, const wg_buffer *A, int64_t offA,
                   int64_t lda, const wg_buffer *x, int64_t offx, int64_t incx, double beta, wg_buffer *y,
                   int64_t offy, int64_t incy, float *gpu_ms);
/* The same on raw device pointers of the device (no size checks). */
wg_status wg_sgemv_dev(wg_device *dev, int trans, int64_t m, int64_t n, float alpha, const float *A, int64_t lda,
                       const float *x, int64_t incx, float beta, float *y, int64_t incy);
wg_status wg_dgemv_dev(wg_device *dev, int trans, int64_t m, int64_t n, double alpha, const double *A, int64_t lda,
                       const double *x, int64_t incx, double beta, double *y, int64_t incy);

/* ---- multi-GPU: C sharded by row blocks, B broadcast over NVLink (NCCL) ---- */
/* The reference drives several GPUs only as independent devices with no data
 * exchange (src/init.mjs:14-29, examples/init-two-gpus/init-two-gpus.js); this
 * adds the sharded GEMM of its multi-GPU target. One communicator per device
 * handle (one process per GPU, or one handle per GPU in a process). NCCL is
 * loaded at run time (libnccl.so.2). */
typedef struct wg_comm wg_comm;
#define WG_COMM_ID_BYTES 128
/* A fresh communicator id; rank 0 makes it and shares it out of band. */
wg_status wg_comm_unique_id(unsigned char *id, size_t len);
/* Joins communicator `id` as `rank` of `nranks`. Non-blocking init: gives up
 * after timeout_ms (<= 0: 60 s), aborting, with WG_ERR_NCCL. */
wg_status wg_comm_init_rank(wg_device *dev, int nranks, int rank, const unsigned char *id, size_t len,
                            int timeout_ms, wg_comm **out);
wg_status wg_comm_destroy(wg_comm *comm);
wg_status wg_comm_abort(wg_comm *comm);
wg_status wg_comm_rank(const wg_comm *comm, int *rank, int *nranks);
/* Waits (bounded by the communicator's timeout) for the last sharded call's
 * work; on timeout or an asynchronous NCCL error aborts and returns WG_ERR_NCCL. */
wg_status wg_comm_wait(wg_comm *comm);
/* This rank's block of C (m_local x n, device pointer, ldc) := alpha * op(A_local)
 * (m_local x k) * op(B) + beta * C_local. B (column-major k x n, or n x k when
 * transB, leading dimension ldb) is read on `root` only; it may be NULL on the
 * other ranks, which receive root's B into the communicator's own buffer. B is
 * sent in column panels (panel_cols wide; <= 0: the planned widths of
 * wg_sharded_panel_plan for an sgemm with k >= 64 and transB = 0, else one
 * panel), and the GEMM of each panel starts as soon as that panel has arrived.
 * n, k, ldb, transB, root and panel_cols must agree on every rank. Queued on the
 * device stream; wg_comm_wait or wg_device_sync waits for it. */
wg_status wg_sgemm_sharded(wg_comm *comm, int transA, int transB, int64_t m_local, int64_t n, int64_t k,
                           float alpha, const float *A_local, int64_t lda, float *B, int64_t ldb, int root,
                           float beta, float *C_local, int64_t ldc, int64_t panel_cols);
wg_status wg_dgemm_sharded(wg_comm *comm, int transA, int transB, int64_t m_local, int64_t n, int64_t k,
                           double alpha, const double *A_local, int64_t lda, double *B, int64_t ldb, int root,
                           double beta, double *C_local, int64_t ldc, int64_t panel_cols);
/* Gathers every rank's C rows into C_full (ldc_full) on `root`; row_offsets has
 * nranks+1 entries (rank r owns rows [row_offsets[r], row_offsets[r+1])). */
wg_status wg_sgemm_gather_rows(wg_comm *comm, const float *C_local, int64_t m_local, int64_t n, int64_t ldc,
                               int root, float *C_full, int64_t ldc_full, const int64_t *row_offsets);
wg_status wg_dgemm_gather_rows(wg_comm *comm, const double *C_local, int64_t m_local, int64_t n, int64_t ldc,
                               int root, double *C_full, int64_t ldc_full, const int64_t *row_offsets);

/* ---- seeded inputs: src/random/random.mjs:4-26 ------------------------------ */
/* randomFloat32Array(n, low, high, seed) / randomFloat64Array: mulberry32 draws
 * u in [0, 1), out[i] = low + u*(high-low) formed in double. */
void wg_random_f32(float *out, int64_t n, double low, double high, uint32_t seed);
void wg_random_f64(double *out, int64_t n, double low, double high, uint32_t seed);
/* Standard normal draws: Box-Muller over the same mulberry32 stream (an
 * addition; the reference has no normal generator). */
void wg_random_normal_f32(float *out, int64_t n, uint32_t seed);
void wg_random_normal_f64(double *out, int64_t n, uint32_t seed);

#ifdef __cplusplus
}
#endif
#endif /* WGBLAS_H */
