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
  WG_DW_FALLBACK = 1,     // epoch of the latest sgemm call whose operands ruled out 3xTF32
  WG_DW_FALLBACKS = 2,    // number of FFMA fallbacks run because a gate was open
  WG_DW_FALLBACK_A = 3,   // panelled products: epoch of the latest op(A) that ruled out 3xTF32
  WG_DW_FALLBACK_B0 = 4,  // panelled products: the same for the op(B) panels of split buffer 0
  WG_DW_FALLBACK_B1 = 5,  // ... and of split buffer 1
  WG_DW_NEXT_UNIT0 = 6,   // work counter of the 3xTF32 kernel (single calls, products' buffer 0)
  WG_DW_NEXT_UNIT1 = 7,   // ... of products' split buffer 1
  WG_DW_COUNT = 8
};

// Device-side switch between the 3xTF32 kernel and its FFMA fallback: open
// (fall back) when *a == ea or *b == eb. The operand split sets the words; a
// tensor-core launch exits at once when its gate is open, and the FFMA launch
// queued after it runs only then.
struct wg_gate {
  const unsigned *a, *b;
  uint32_t ea, eb;
};

// The triangle of an m x n C that gemmtr-style calls update, in the column-major
// frame: WG_UPLO_FULL every element, WG_UPLO_LOWER C(i, j) with j <= i,
// WG_UPLO_UPPER j >= i (src/shaders/sgemm_large.wgsl:293-297).
#ifdef __CUDACC__
__host__ __device__
#endif
inline bool wg_in_triangle(int uplo, int64_t i, int64_t j) {
  return uplo == WG_UPLO_FULL || (uplo == WG_UPLO_LOWER ? j <= i : j >= i);
}
// True when no element of the block [i0, i0 + h) x [j0, j0 + w) is in the triangle
// (such a tile is skipped: src/shaders/sgemm_large.wgsl:78-83).
#ifdef __CUDACC__
__host__ __device__
#endif
inline bool wg_tile_outside(int uplo, int64_t i0, int64_t h, int64_t j0, int64_t w) {
  return (uplo == WG_UPLO_LOWER && j0 > i0 + h - 1) || (uplo == WG_UPLO_UPPER && j0 + w - 1 < i0);
}
#ifdef __CUDACC__
// Programmatic dependent launch. A kernel launched with programmatic stream
// serialization may start once every CTA of the kernel before it in the stream
// has run wg_pdl_trigger (or exited); wg_pdl_wait then blocks until that kernel
// has completed and its memory operations are visible. Without the launch
// attribute the wait returns at once.
__device__ __forceinline__ void wg_pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void wg_pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ bool wg_gate_open(const wg_gate &g) {
  return *(volatile const unsigned *)g.a == g.ea || *(volatile const unsigned *)g.b == g.eb;
}
#endif
// Bits of WG_DW_ERROR.
enum {
  WG_DERR_TMA_WAIT = 1u,  // producer or consumer gave up waiting on a pipeline stage
  WG_DERR_MMA_WAIT = 2u,  // the epilogue gave up waiting for the accumulator
  WG_DERR_TMEM = 4u,      // TMEM allocation returned an unusable address
  WG_DERR_SELFTEST = 8u,  // wg_selftest_bounded_wait's wait ran out, as it is meant to
  WG_DERR_FLOW_WAIT = 16u  // a strsm flow CTA gave up waiting for an earlier block
};

struct wg_device {
  int ordinal;
  unsigned flags;
  cudaStream_t own_stream;
  cudaStream_t stream;  // the stream work is ordered on (own_stream or the caller's)
  cudaEvent_t ev_start, ev_stop;
  int sm_count;
  int cc_major, cc_minor;
  size_t total_mem;
  char name[256];
  void *ws;          // grow-only scratch for the 3xTF32 operand split
  size_t ws_bytes;
  unsigned *dwords;  // WG_DW_COUNT device words
  uint32_t epoch;    // sgemm call counter, tags WG_DW_FALLBACK
  int sgemm_path;
  int dgemm_path;
  int fused_bn;  // tile width forced on the fused 3xTF32 kernel (0: chosen per call)
  int strsm_path;
  // strsm flow: per (right-hand-side chunk, 64-row block) "solved" words,
  // written only by the flow kernel with the call's epoch (zero when allocated)
  unsigned *flow_flags;
  size_t flow_flags_n;
  uint32_t flow_epoch;
  cudaStream_t h2d, d2h;  // copy streams of the host-array path (created on first use)
  cudaMemPool_t staging;  // device copies of host-array operands; keeps its memory between calls
  // panelled 3xTF32 products: the stream their operand splits run on, and events
  // (entry, op(A) split ready, a panel's op(B) split ready, split buffer 0/1 free)
  cudaStream_t side;
  cudaEvent_t tc_ev[5];
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
// Counts one kernel launch and, while profiling is on, brackets it with events
// on the stream it is launched on (the device stream unless given).
struct wg_launch_scope {
  wg_device *d;
  cudaStream_t s;
  int slot;
  wg_launch_scope(wg_device *dev, const char *family) : wg_launch_scope(dev, family, nullptr) {}
  wg_launch_scope(wg_device *dev, const char *family, cudaStream_t stream);
  ~wg_launch_scope();
};

struct wg_buffer {
  wg_device *dev;
  void *ptr;
  size_t bytes;
  int pooled;  // memory from the device's stream-ordered pool (wg_buffer_alloc_async)
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

// Raises kernel `fn`'s dynamic shared-memory limit to `bytes` (and, when asked,
// its preferred carveout to the maximum) on the current device, once per
// (kernel, device, bytes): the attributes last for the context, and setting
// them again on every launch put host time between the caller's stream
// operations. (runtime.cu)
cudaError_t wg_kernel_smem_raw(const void *fn, size_t bytes, bool max_carveout);
template <class F>
cudaError_t wg_kernel_smem(F *fn, size_t bytes, bool max_carveout = false) {
  return wg_kernel_smem_raw(reinterpret_cast<const void *>(fn), bytes, max_carveout);
}

// Launches `kern` with programmatic stream serialization: it may be scheduled
// while the kernel before it on the stream finishes, so it must call
// wg_pdl_wait before it touches memory (gemv.cu, which also triggers its own
// dependents right after that wait).
template <class... KArgs, class... Args>
cudaError_t wg_launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                          Args &&...args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<Args &&>(args)...);
}

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
                          const T *A, int64_t lda, const T *B, int64_t ldb, T beta, T *C, int64_t ldc, int uplo = 0);

// One column panel (cols columns) of a product queued panel by panel on
// d->stream, through the dispatcher (sgemm products on the tensor cores use
// wg_tc_product instead).
template <typename T>
wg_status wg_gemm_panel(wg_device *d, int transA, int transB, int64_t m, int64_t cols, int64_t k, T alpha,
                        const T *A, int64_t lda, const T *B, int64_t ldb, T beta, T *C, int64_t ldc);
// True when an sgemm panel of this shape can run on the 3xTF32 kernel.
bool wg_sgemm_panel_on_tc(const wg_device *d, float alpha, int64_t m, int64_t cols, int64_t k);

// A 3xTF32 sgemm computed in column panels whose op(B) arrives panel by panel
// (uploaded from the host, or broadcast from another GPU). op(A) is split once;
// each panel's op(B) is split on the device's side stream into one of two
// alternating buffers, so the split of panel j+1 runs while the MMA of panel j
// runs on d->stream. Each split flags its own operand (WG_DW_FALLBACK_A, _B0/_B1
// with a fresh epoch), and a panel whose op(A) or op(B) is ruled out runs on
// the FFMA kernel instead, so one bad panel does not send the others there.
struct wg_tc_product {
  wg_device *d;
  int transA, transB;
  int64_t m, k;
  float alpha, beta;
  const float *A;
  int64_t lda;
  char *ws;
  size_t a_region, slot_bytes, partial_room;
  int64_t counter_room;
  int64_t panels;
  uint32_t epoch_a;
  bool fused;       // panels run on the fused kernel (no operand splits, no side stream)
  size_t ws_bytes;  // the fused panels' scratch
};
// Scratch of a product with these panel widths (queried before begin).
size_t wg_tc_product_workspace(const wg_device *d, int64_t m, int64_t k, const int64_t *widths, size_t count);
// Starts a product; every later panel must be one of `widths`. B0 / ldb: the
// stored B the panels are cut from (its base and leading dimension). When the
// fused kernel can read op(A) and every panel of op(B) (16-byte aligned bases,
// leading dimensions multiples of 4), each panel is one fused launch on
// d->stream after its b_ready event (a_ready then orders the first one).
// Otherwise op(A) is split here (on the side stream, after a_ready when given).
wg_status wg_tc_product_begin(wg_tc_product *p, wg_device *d, int transA, int transB, int64_t m, int64_t k,
                              float alpha, const float *A, int64_t lda, float beta, const int64_t *widths,
                              size_t count, cudaEvent_t a_ready, const float *B0, int64_t ldb);
// C (m x cols) = alpha*op(A)*op(B panel) + beta*C once b_ready (when given) has
// fired: the split on the side stream, the MMA and its gated FFMA fallback on
// d->stream. B is the panel's first column of op(B) in the caller's layout.
wg_status wg_tc_product_panel(wg_tc_product *p, int64_t cols, const float *B, int64_t ldb, float *C, int64_t ldc,
                              cudaEvent_t b_ready);
// Orders d->stream after everything the product queued on the side stream (call
// it before releasing operands the splits read, also after an error).
void wg_tc_product_join(wg_tc_product *p);

// Returns at least `bytes` of device scratch owned by the handle (stream-ordered reuse).
wg_status wg_workspace(wg_device *dev, size_t bytes, void **ptr);
// The device's stream-ordered memory pool (created on first use, destroyed
// with the handle). It keeps the memory it has mapped when allocations are
// freed, so repeated temporaries of the same sizes cost no mapping.
wg_status wg_staging_pool(wg_device *dev);

// ---- kernel launchers (gemm_simt.cu, sgemm_tf32x3.cu) ----

// The same FFMA arithmetic on 32 x 64 tiles (small products: every SM gets a tile).
cudaError_t wg_launch_gemm_simt_small(cudaStream_t s, int transA, int transB, int64_t m, int64_t n, int64_t k,
                                      float alpha, const float *A, int64_t lda, const float *B, int64_t ldb,
                                      float beta, float *C, int64_t ldc, int uplo);
// C = alpha*op(A)op(B) + beta*C on the FFMA / DFMA pipes, sequential k per element.
// With a gate, every CTA first checks it and exits unless it is open (the
// device-side fallback of the 3xTF32 path), counting runs in dwords[WG_DW_FALLBACKS].
template <typename T>
cudaError_t wg_launch_gemm_simt(cudaStream_t s, int transA, int transB, int64_t m, int64_t n,
                                int64_t k, T alpha, const T *A, int64_t lda, const T *B,
                                int64_t ldb, T beta, T *C, int64_t ldc, unsigned *dwords,
                                const wg_gate *gate, int uplo = 0);

// Which columns of a gated FFMA launch to compute: those of the fused 3xTF32
// kernel's tiles (tiles_m x ..., tile width bn, 128 rows) whose flag holds epoch.
struct wg_tile_mask {
  const unsigned *flags;
  int tiles_m, bn;
  uint32_t epoch;
};
// The gated FFMA launch restricted to the flagged tiles of a fused 3xTF32 call.
template <typename T>
cudaError_t wg_launch_gemm_simt_masked(cudaStream_t s, int transA, int transB, int64_t m, int64_t n, int64_t k,
                                       T alpha, const T *A, int64_t lda, const T *B, int64_t ldb, T beta, T *C,
                                       int64_t ldc, unsigned *dwords, const wg_gate *gate, const wg_tile_mask *mask,
                                       int uplo = 0);

// The fused 3xTF32 kernel (sgemm_fused.cu): op(A), op(B) read by TMA straight
// from the caller's matrices and split inside the kernel. Supported when both
// bases are 16-byte aligned and lda, ldb are multiples of 4. Chosen
// automatically for products of at most WG_FUSED_MAX_WORK multiply-adds: there
// it saves the split pass and its launch; on larger ones its in-kernel split
// competes with the MMAs for shared-memory bandwidth (measured on B200: 0.92
// ms against 0.61 ms for the split pass + MMA kernel at 4096^3).
constexpr double WG_FUSED_MAX_WORK = 1.2e9;
bool wg_tf32x3_fused_supported(const wg_device *d, int transA, int transB, int64_t m, int64_t n, int64_t k,
                               const float *A, int64_t lda, const float *B, int64_t ldb);
// Scratch one fused call needs (split-K partial sums, counters, tile flags).
size_t wg_tf32x3_fused_workspace(const wg_device *d, int64_t m, int64_t n, int64_t k);
// The CTA-pair form of the fused kernel (256 x 256 tiles, tcgen05 cta_group::2):
// its scratch, and the call (the kernel and its gated FFMA fallback on stream
// st). Same support rule as the fused kernel; runs when WG_SGEMM_TF32X3_PAIR is
// set (measured on B200 at 4096^3: 1.02 ms, against 0.82 ms for the one-CTA
// fused kernel and 0.61 ms for the split pass + MMA kernel).
size_t wg_tf32x3_pair_workspace(const wg_device *d, int64_t m, int64_t n, int64_t k);
wg_status wg_sgemm_tf32x3_pair(wg_device *d, cudaStream_t st, int transA, int transB, int64_t m, int64_t n, int64_t k,
                               float alpha, const float *A, int64_t lda, const float *B, int64_t ldb, float beta,
                               float *C, int64_t ldc, void *ws, size_t ws_bytes, int uplo = 0);
// Queues the fused kernel and its gated FFMA fallback on stream st.
wg_status wg_sgemm_tf32x3_fused(wg_device *d, cudaStream_t st, int transA, int transB, int64_t m, int64_t n,
                                int64_t k, float alpha, const float *A, int64_t lda, const float *B, int64_t ldb,
                                float beta, float *C, int64_t ldc, void *ws, size_t ws_bytes, int uplo = 0);

// dgemm on the FP64 tensor-core (DMMA) path (dgemm_dmma.cu), on d->stream: the
// TMA-fed pipelined kernel when the operands' layout allows its tensor maps,
// the register-staged kernel otherwise.
wg_status wg_dgemm_dmma(wg_device *d, int transA, int transB, int64_t m, int64_t n, int64_t k, double alpha,
                        const double *A, int64_t lda, const double *B, int64_t ldb, double beta, double *C,
                        int64_t ldc, int uplo = 0);

// cuTensorMapEncodeTiled, reached through the runtime's driver entry point (no
// link-time dependency on libcuda); NULL when the driver does not provide it.
#include <cuda.h>
typedef CUresult (*wg_encode_tiled_fn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                       const cuuint64_t *, const cuuint32_t *, const cuuint32_t *,
                                       CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                       CUtensorMapFloatOOBfill);
wg_encode_tiled_fn wg_encode_tiled();

// C = (alpha == 0 ? 0 : alpha*0) + beta*C elementwise — the k == 0 / alpha == 0 cases.
template <typename T>
cudaError_t wg_launch_scale(cudaStream_t s, int64_t m, int64_t n, T alpha, T beta, T *C,
                            int64_t ldc, int uplo = 0);

// Bytes of scratch the 3xTF32 path needs for this shape: the split operands
// alone (whole-tile scheduling), or with the split-K partial sums and counters.
size_t wg_tf32x3_workspace_bytes(int64_t m, int64_t n, int64_t k);
size_t wg_tf32x3_workspace_bytes_sk(const wg_device *dev, int64_t m, int64_t n, int64_t k);
// Modelled run time of the 3xTF32 kernel for one m x n x k product on G SMs, in
// units of one 16-deep k-block of one tile's MMAs (about 0.5 us on B200).
double wg_tf32x3_cost(int G, int64_t m, int64_t n, int64_t k);
// True when the 3xTF32 path supports this shape on this device.
bool wg_tf32x3_supported(const wg_device *dev, int64_t m, int64_t n, int64_t k);
// Looks up (and so reserves) wg_sgemm_noalloc's fixed scratch on a device; called
// when a handle is opened. A failure is left for the first wg_sgemm_noalloc call.
void wg_noalloc_reserve(int ordinal);
// Splits op(A), op(B) into tf32 hi/lo operands in `ws`, then runs the tcgen05 kernel.
// Operands outside the split's exact range make the kernel exit and the FFMA
// kernel (launched right after, gated on the same epoch) compute C instead.
// `ws` holds ws_bytes: the last wave is split along k when it also fits the
// partial sums (wg_tf32x3_workspace_bytes_sk), whole tiles otherwise.
wg_status wg_sgemm_tf32x3(wg_device *dev, int transA, int transB, int64_t m, int64_t n,
                          int64_t k, float alpha, const float *A, int64_t lda, const float *B,
                          int64_t ldb, float beta, float *C, int64_t ldc, void *ws, size_t ws_bytes, int uplo = 0);
uint32_t wg_next_epoch(wg_device *dev);
