// Multi-GPU sgemm / dgemm: C sharded by row blocks across ranks, the shared
// operand B broadcast over NVLink with NCCL, one process (or device handle)
// per GPU.
//
// The reference has no multi-GPU exchange at all (several independent
// GPUDevices, src/init.mjs:14-29); this is the sharding the north star asks
// for. Rank r owns rows [off_r, off_r + m_r) of C and of op(A), resident on its
// GPU (scattered once). Each call broadcasts B from `root` in column panels on
// the communicator's stream; the GEMM of panel j on the device stream waits
// only for panel j's broadcast, so the transfer of panel j+1 overlaps the math
// of panel j. Every kernel reads only its own GPU's memory: remote data
// arrives through NCCL into local buffers (no peer loads, no TMA multicast).
//
// NCCL (libnccl.so.2) is opened at run time, so the library loads on machines
// without it and shares the copy a host framework already loaded. The
// communicator is created non-blocking and every wait on it is bounded by a
// host timeout after which the communicator is aborted and WG_ERR_NCCL is
// returned, so a rank that never joins or dies surfaces as an error instead
// of a hang.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <new>
#include <mutex>
#include <thread>
#include <type_traits>
#include <vector>

#include "internal.h"

namespace {

struct NcclApi {
  bool ok = false;
  ncclResult_t (*GetUniqueId)(ncclUniqueId *);
  ncclResult_t (*CommInitRankConfig)(ncclComm_t *, int, ncclUniqueId, int, ncclConfig_t *);
  ncclResult_t (*CommDestroy)(ncclComm_t);
  ncclResult_t (*CommAbort)(ncclComm_t);
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t *);
  ncclResult_t (*Broadcast)(const void *, void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
  ncclResult_t (*AllReduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t);
  ncclResult_t (*Send)(const void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
  ncclResult_t (*Recv)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t);
  ncclResult_t (*GroupStart)();
  ncclResult_t (*GroupEnd)();
  const char *(*GetErrorString)(ncclResult_t);
};

NcclApi *nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
#define LOAD(field, sym) api.field = reinterpret_cast<decltype(api.field)>(dlsym(h, sym))
    LOAD(GetUniqueId, "ncclGetUniqueId");
    LOAD(CommInitRankConfig, "ncclCommInitRankConfig");
    LOAD(CommDestroy, "ncclCommDestroy");
    LOAD(CommAbort, "ncclCommAbort");
    LOAD(CommGetAsyncError, "ncclCommGetAsyncError");
    LOAD(Broadcast, "ncclBroadcast");
    LOAD(AllReduce, "ncclAllReduce");
    LOAD(Send, "ncclSend");
    LOAD(Recv, "ncclRecv");
    LOAD(GroupStart, "ncclGroupStart");
    LOAD(GroupEnd, "ncclGroupEnd");
    LOAD(GetErrorString, "ncclGetErrorString");
#undef LOAD
    api.ok = api.GetUniqueId && api.CommInitRankConfig && api.CommDestroy && api.CommAbort &&
             api.CommGetAsyncError && api.Broadcast && api.AllReduce && api.Send && api.Recv && api.GroupStart && api.GroupEnd &&
             api.GetErrorString;
  });
  return api.ok ? &api : nullptr;
}

}  // namespace

struct wg_comm {
  wg_device *dev;
  ncclComm_t comm;
  int nranks, rank;
  cudaStream_t stream;          // the communicator's stream (broadcast panels)
  std::vector<cudaEvent_t> ev;  // panel-ready events, reused call to call
  cudaEvent_t entry;            // the device stream at entry (B ready, previous readers done)
  cudaEvent_t done;             // all of the call's work, for bounded waits
  int timeout_ms;
  bool aborted;
  // Last automatic panel plan, keyed by (n, k): planning a very wide product
  // is not free, and the ranks must agree on the widths (see agreed_panels).
  int64_t plan_key[2];
  std::vector<int64_t> plan_widths;
  int64_t *agree;       // two device words for the planning all-reduce
  int64_t *agree_host;  // and their page-locked host copy
  cudaEvent_t agreed;
};

namespace {

wg_status nccl_fail(wg_comm *c, ncclResult_t r, const char *what) {
  NcclApi *N = nccl();
  return wg_fail(WG_ERR_NCCL, "%s failed: %s (rank %d of %d)", what, N ? N->GetErrorString(r) : "NCCL missing",
                 c ? c->rank : -1, c ? c->nranks : 0);
}

// Waits while the non-blocking communicator reports ncclInProgress.
wg_status settle(wg_comm *c, ncclResult_t r, const char *what) {
  NcclApi *N = nccl();
  const auto t0 = std::chrono::steady_clock::now();
  while (r == ncclInProgress) {
    if (std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(c->timeout_ms)) {
      N->CommAbort(c->comm);
      c->aborted = true;
      return wg_fail(WG_ERR_NCCL, "%s did not complete within %d ms on rank %d; communicator aborted", what,
                     c->timeout_ms, c->rank);
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
    N->CommGetAsyncError(c->comm, &r);
  }
  if (r != ncclSuccess) return nccl_fail(c, r, what);
  return WG_OK;
}

// Waits for `ev` (recorded on the communicator's stream), bounded by the
// communicator's timeout; aborts the communicator on timeout or an
// asynchronous NCCL error.
wg_status wait_event(wg_comm *c, cudaEvent_t ev, const char *what) {
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    cudaError_t e = cudaEventQuery(ev);
    if (e == cudaSuccess) return WG_OK;
    if (e != cudaErrorNotReady) return wg_fail(WG_ERR_CUDA, "%s failed: %s", what, cudaGetErrorString(e));
    ncclResult_t r = ncclSuccess;
    nccl()->CommGetAsyncError(c->comm, &r);
    if ((r != ncclSuccess && r != ncclInProgress) ||
        std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(c->timeout_ms)) {
      nccl()->CommAbort(c->comm);
      c->aborted = true;
      return r != ncclSuccess && r != ncclInProgress
                 ? nccl_fail(c, r, what)
                 : wg_fail(WG_ERR_NCCL, "%s did not finish within %d ms on rank %d; communicator aborted", what,
                           c->timeout_ms, c->rank);
    }
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
}

template <typename T>
ncclDataType_t nccl_type();
template <>
ncclDataType_t nccl_type<float>() { return ncclFloat; }
template <>
ncclDataType_t nccl_type<double>() { return ncclDouble; }

// Frees the communicator's CUDA resources (whichever were created) and the
// object itself; the NCCL communicator is destroyed or aborted by the caller.
void release(wg_comm *c) {
  for (cudaEvent_t e : c->ev) cudaEventDestroy(e);
  if (c->entry) cudaEventDestroy(c->entry);
  if (c->done) cudaEventDestroy(c->done);
  if (c->agreed) cudaEventDestroy(c->agreed);
  if (c->agree) cudaFree(c->agree);
  if (c->agree_host) cudaFreeHost(c->agree_host);
  if (c->stream) cudaStreamDestroy(c->stream);
  delete c;
}

cudaEvent_t panel_event(wg_comm *c, size_t i) {
  while (c->ev.size() <= i) {
    cudaEvent_t e = nullptr;
    cudaEventCreateWithFlags(&e, cudaEventDisableTiming);
    c->ev.push_back(e);
  }
  return c->ev[i];
}

// Column panels of a sharded sgemm on the 3xTF32 kernel. Panel j's GEMM starts
// when both the previous panel's GEMM and panel j's broadcast are done; with
// the broadcast of consecutive panels back to back on the communicator's
// stream, the end time of the product is a shortest path over the panel
// boundaries, found here by dynamic programming over 256-column tile columns.
// Costs are in units of one 16-deep k-block of one tile's MMAs (about 0.5 us):
// the GEMM from the kernel's own schedule model (wg_tf32x3_cost), the B split
// at about 5 TB/s (4 bytes read, 8 written per element), about 30 us per panel
// for its three launches and the pipeline fill and drain, and the broadcast at
// about 400 GB/s when there is more than one rank. Wave quantisation makes
// the panel widths matter: 16 tile rows x 9 tile columns fill 144 of 148 SMs,
// 16 x 8 only 128.
std::vector<int64_t> plan_panels(int G, int nranks, int64_t m, int64_t n, int64_t k) {
  constexpr double kb_s = 0.5e-6;
  constexpr double kPanelFixed = 60.0;
  const int64_t tc = (n + 255) / 256;
  const int64_t cmax = tc < 256 ? tc : 256;
  const double kp = (double)((k + 31) / 32 * 32);
  const double bcast = nranks > 1 ? 256.0 * (double)k * 4.0 / 400e9 / kb_s : 0.0;  // per tile column
  const double pack = 256.0 * kp * 12.0 / 5e12 / kb_s;
  std::vector<double> full(cmax + 1, 0.0);  // GEMM cost of a panel of c whole tile columns
  for (int64_t c = 1; c <= cmax; c++) full[c] = wg_tf32x3_cost(G, m, c * 256, k);
  std::vector<double> best(tc + 1, 1e300);
  std::vector<int64_t> from(tc + 1, 0);
  best[0] = 0.0;
  for (int64_t y = 1; y <= tc; y++) {
    for (int64_t c = 1; c <= cmax && c <= y; c++) {
      const int64_t x = y - c;
      const int64_t cols = (y * 256 < n ? y * 256 : n) - x * 256;
      const double gemm = cols == c * 256 ? full[c] : wg_tf32x3_cost(G, m, cols, k);
      const double arrive = (double)y * bcast;  // panel [x, y) fully broadcast
      const double t = (best[x] > arrive ? best[x] : arrive) + (double)c * pack + gemm + kPanelFixed;
      if (t < best[y]) {
        best[y] = t;
        from[y] = x;
      }
    }
  }
  std::vector<int64_t> widths;
  for (int64_t y = tc; y > 0; y = from[y]) widths.push_back((y * 256 < n ? y * 256 : n) - from[y] * 256);
  return std::vector<int64_t>(widths.rbegin(), widths.rend());
}

// The automatic panel widths of a sharded sgemm. Every rank must broadcast the
// same panels, so the plan is made only from values all ranks share: n, k and
// the rank count, plus the largest m_local and the fewest SMs of any rank,
// agreed by one all-reduce. The plan is cached per (n, k); the ranks make their
// calls with the same (n, k) sequence, so they take the all-reduce together.
wg_status agreed_panels(wg_comm *c, int64_t m_local, int64_t n, int64_t k, std::vector<int64_t> &out) {
  if (!c->plan_widths.empty() && c->plan_key[0] == n && c->plan_key[1] == k) {
    out = c->plan_widths;
    return WG_OK;
  }
  int64_t m_max = m_local, g_min = c->dev->sm_count;
  if (c->nranks > 1) {
    c->agree_host[0] = m_local;
    c->agree_host[1] = -g_min;
    WG_CUDA(cudaMemcpyAsync(c->agree, c->agree_host, 2 * sizeof(int64_t), cudaMemcpyHostToDevice, c->stream));
    wg_status st = settle(c, nccl()->AllReduce(c->agree, c->agree, 2, ncclInt64, ncclMax, c->comm, c->stream),
                          "ncclAllReduce");
    if (st != WG_OK) return st;
    WG_CUDA(cudaMemcpyAsync(c->agree_host, c->agree, 2 * sizeof(int64_t), cudaMemcpyDeviceToHost, c->stream));
    WG_CUDA(cudaEventRecord(c->agreed, c->stream));
    st = wait_event(c, c->agreed, "panel planning all-reduce");
    if (st != WG_OK) return st;
    m_max = c->agree_host[0];
    g_min = -c->agree_host[1];
  }
  c->plan_widths = m_max > 0 && g_min > 0 ? plan_panels((int)g_min, c->nranks, m_max, n, k)
                                          : std::vector<int64_t>{n};
  c->plan_key[0] = n;
  c->plan_key[1] = k;
  out = c->plan_widths;
  return WG_OK;
}

template <typename T>
wg_status sharded(wg_comm *c, int transA, int transB, int64_t m_local, int64_t n, int64_t k, T alpha, const T *A,
                  int64_t lda, T *B, int64_t ldb, int root, T beta, T *C, int64_t ldc, int64_t panel) {
  if (!c || c->aborted) return wg_fail(WG_ERR_INVALID_ARGUMENT, "communicator is NULL or aborted");
  if ((transA | transB) & ~1) return wg_fail(WG_ERR_INVALID_ARGUMENT, "trans flags must be 0 or 1");
  if (m_local < 0 || n < 0 || k < 0) return wg_fail(WG_ERR_INVALID_ARGUMENT, "m, n, and k must be non-negative.");
  if (root < 0 || root >= c->nranks) return wg_fail(WG_ERR_INVALID_ARGUMENT, "root %d out of range", root);
  if (ldb < (transB ? n : k) || ldb <= 0 || lda <= 0 || ldc <= 0 || ldc < m_local || lda < (transA ? k : m_local))
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "a leading dimension is below the rows of its matrix as stored");
  if (n == 0 || k == 0 || !B) {
    // Nothing to broadcast; each rank scales its own block (k == 0) or has nothing to do.
    if (m_local && n) return wg_gemm_enqueue<T>(c->dev, transA, transB, m_local, n, k, alpha, A, lda, B, ldb, beta,
                                                C, ldc);
    return WG_OK;
  }
  NcclApi *N = nccl();
  wg_device *d = c->dev;
  wg_device_guard guard(d->ordinal);
  // Panel widths, the same on every rank: one panel for a transposed B (its
  // columns are not contiguous), the caller's width when given, planned widths
  // for an sgemm the 3xTF32 kernel can take, else one panel.
  std::vector<int64_t> widths;
  const bool auto_plan = std::is_same<T, float>::value && !transB && panel <= 0 && alpha != T(0) && k >= 64;
  if (transB || (panel <= 0 && !auto_plan)) {
    widths.push_back(n);
  } else if (panel > 0) {
    for (int64_t j0 = 0; j0 < n; j0 += panel) widths.push_back(n - j0 < panel ? n - j0 : panel);
  } else {
    wg_status st = agreed_panels(c, m_local, n, k, widths);
    if (st != WG_OK) return st;
  }
  int64_t widest = 0;
  for (int64_t w : widths) widest = w > widest ? w : widest;
  // This rank's panels run on the 3xTF32 kernel when its own block allows it.
  const bool tc = std::is_same<T, float>::value && m_local > 0 && !transB &&
                  wg_sgemm_panel_on_tc(d, (float)alpha, m_local, widest, k);
  // B must be ready on root, and earlier readers of B done on every rank, before it is overwritten.
  WG_CUDA(cudaEventRecord(c->entry, d->stream));
  WG_CUDA(cudaStreamWaitEvent(c->stream, c->entry, 0));
  // On the tensor cores the panels form one product: op(A) is split once, and
  // each arriving panel's split overlaps the previous panel's MMA.
  wg_tc_product prod{};
  wg_status st = WG_OK;
  if (tc)
    st = wg_tc_product_begin(&prod, d, transA, transB, m_local, k, (float)alpha, (const float *)A, lda, (float)beta,
                             widths.data(), widths.size(), nullptr);
  int64_t j0 = 0;
  for (size_t j = 0; st == WG_OK && j < widths.size(); j++) {
    const int64_t cols = widths[j];
    // Column panel of a column-major k x n B (transB = 0), or all of the n x k B.
    const size_t count = transB ? (size_t)((k - 1) * ldb + n) : (size_t)((cols - 1) * ldb + k);
    T *bp = B + (transB ? 0 : j0 * ldb);
    st = settle(c, N->Broadcast(bp, bp, count, nccl_type<T>(), root, c->comm, c->stream), "ncclBroadcast");
    if (st != WG_OK) break;
    cudaEvent_t ev = panel_event(c, j);
    cudaError_t e = cudaEventRecord(ev, c->stream);
    if (e != cudaSuccess) {
      st = wg_fail(WG_ERR_CUDA, "cudaEventRecord failed: %s", cudaGetErrorString(e));
      break;
    }
    T *cp = C + (transB ? 0 : j0 * ldc);
    if (tc) {
      st = wg_tc_product_panel(&prod, cols, (const float *)bp, ldb, (float *)cp, ldc, ev);
    } else {
      e = cudaStreamWaitEvent(d->stream, ev, 0);
      if (e != cudaSuccess) st = wg_fail(WG_ERR_CUDA, "cudaStreamWaitEvent failed: %s", cudaGetErrorString(e));
      else if (m_local > 0)
        st = wg_gemm_panel<T>(d, transA, transB, m_local, cols, k, alpha, A, lda, bp, ldb, beta, cp, ldc);
    }
    j0 += cols;
  }
  if (tc) wg_tc_product_join(&prod);
  if (st != WG_OK) return st;
  WG_CUDA(cudaEventRecord(c->done, d->stream));
  return WG_OK;
}

template <typename T>
wg_status gather(wg_comm *c, const T *C_local, int64_t m_local, int64_t n, int64_t ldc, int root, T *C_full,
                 int64_t ldc_full, const int64_t *row_offsets) {
  if (!c || c->aborted) return wg_fail(WG_ERR_INVALID_ARGUMENT, "communicator is NULL or aborted");
  if (!row_offsets || root < 0 || root >= c->nranks) return wg_fail(WG_ERR_INVALID_ARGUMENT, "invalid argument");
  if (row_offsets[c->rank + 1] - row_offsets[c->rank] != m_local)
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "m_local does not match row_offsets for rank %d", c->rank);
  NcclApi *N = nccl();
  wg_device *d = c->dev;
  wg_device_guard guard(d->ordinal);
  cudaStream_t s = d->stream;  // gathers are ordered after the GEMMs that produce C_local
  const size_t sz = sizeof(T);
  if (c->rank == root) {
    if (!C_full || ldc_full < row_offsets[c->nranks])
      return wg_fail(WG_ERR_INVALID_ARGUMENT, "C_full is NULL or ldc_full is below the total rows");
    int64_t max_rows = 0;
    for (int r = 0; r < c->nranks; r++)
      max_rows = row_offsets[r + 1] - row_offsets[r] > max_rows ? row_offsets[r + 1] - row_offsets[r] : max_rows;
    T *stage = nullptr;
    if (c->nranks > 1 && max_rows && n) WG_CUDA(cudaMallocAsync((void **)&stage, (size_t)max_rows * n * sz, s));
    for (int r = 0; r < c->nranks; r++) {
      const int64_t mr = row_offsets[r + 1] - row_offsets[r];
      if (!mr || !n) continue;
      T *dst = C_full + row_offsets[r];
      if (r == root) {
        WG_CUDA(cudaMemcpy2DAsync(dst, ldc_full * sz, C_local, ldc * sz, mr * sz, n, cudaMemcpyDeviceToDevice, s));
        continue;
      }
      wg_status st = settle(c, N->Recv(stage, (size_t)(mr * n), nccl_type<T>(), r, c->comm, s), "ncclRecv");
      if (st != WG_OK) return st;
      WG_CUDA(cudaMemcpy2DAsync(dst, ldc_full * sz, stage, mr * sz, mr * sz, n, cudaMemcpyDeviceToDevice, s));
    }
    if (stage) cudaFreeAsync(stage, s);
  } else if (m_local && n) {
    const T *src = C_local;
    T *packed = nullptr;
    if (ldc != m_local) {  // rows of a column-major block are strided: send a dense copy
      WG_CUDA(cudaMallocAsync((void **)&packed, (size_t)m_local * n * sz, s));
      WG_CUDA(cudaMemcpy2DAsync(packed, m_local * sz, C_local, ldc * sz, m_local * sz, n, cudaMemcpyDeviceToDevice, s));
      src = packed;
    }
    wg_status st = settle(c, N->Send(src, (size_t)(m_local * n), nccl_type<T>(), root, c->comm, s), "ncclSend");
    if (packed) cudaFreeAsync(packed, s);
    if (st != WG_OK) return st;
  }
  WG_CUDA(cudaEventRecord(c->done, s));
  return WG_OK;
}

}  // namespace

extern "C" wg_status wg_sharded_panel_plan(int sm_count, int nranks, int64_t m_local, int64_t n, int64_t k,
                                           int64_t *widths, size_t capacity, size_t *count) {
  if (!count || sm_count <= 0 || nranks < 1 || m_local <= 0 || n <= 0 || k < 64 || (capacity && !widths))
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "invalid argument");
  const std::vector<int64_t> w = plan_panels(sm_count, nranks, m_local, n, k);
  *count = w.size();
  if (capacity < w.size()) return wg_fail(WG_ERR_INVALID_ARGUMENT, "widths holds %zu, the plan has %zu panels",
                                          capacity, w.size());
  for (size_t i = 0; i < w.size(); i++) widths[i] = w[i];
  return WG_OK;
}

extern "C" wg_status wg_comm_unique_id(unsigned char *id, size_t len) {
  if (!id || len < NCCL_UNIQUE_ID_BYTES) return wg_fail(WG_ERR_INVALID_ARGUMENT, "need a 128-byte id buffer");
  NcclApi *N = nccl();
  if (!N) return wg_fail(WG_ERR_NOT_SUPPORTED, "libnccl.so.2 could not be loaded");
  ncclUniqueId u;
  ncclResult_t r = N->GetUniqueId(&u);
  if (r != ncclSuccess) return wg_fail(WG_ERR_NCCL, "ncclGetUniqueId failed: %s", N->GetErrorString(r));
  memcpy(id, u.internal, NCCL_UNIQUE_ID_BYTES);
  return WG_OK;
}

extern "C" wg_status wg_comm_init_rank(wg_device *d, int nranks, int rank, const unsigned char *id, size_t len,
                                       int timeout_ms, wg_comm **out) {
  if (!d || !out || !id || len < NCCL_UNIQUE_ID_BYTES || nranks < 1 || rank < 0 || rank >= nranks)
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "invalid argument");
  *out = nullptr;
  NcclApi *N = nccl();
  if (!N) return wg_fail(WG_ERR_NOT_SUPPORTED, "libnccl.so.2 could not be loaded");
  wg_device_guard guard(d->ordinal);
  wg_comm *c = new (std::nothrow) wg_comm();
  if (!c) return wg_fail(WG_ERR_OUT_OF_MEMORY, "host allocation failed");
  c->dev = d;
  c->nranks = nranks;
  c->rank = rank;
  c->timeout_ms = timeout_ms > 0 ? timeout_ms : 60000;
  cudaError_t e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c->entry, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c->done, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaEventCreateWithFlags(&c->agreed, cudaEventDisableTiming);
  if (e == cudaSuccess) e = cudaMalloc((void **)&c->agree, 2 * sizeof(int64_t));
  if (e == cudaSuccess) e = cudaHostAlloc((void **)&c->agree_host, 2 * sizeof(int64_t), cudaHostAllocDefault);
  if (e != cudaSuccess) {
    release(c);
    return wg_fail(WG_ERR_CUDA, "communicator stream/event creation failed: %s", cudaGetErrorString(e));
  }
  ncclUniqueId u;
  memcpy(u.internal, id, NCCL_UNIQUE_ID_BYTES);
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclResult_t r = N->CommInitRankConfig(&c->comm, nranks, u, rank, &cfg);
  wg_status st = (r == ncclSuccess || r == ncclInProgress) ? settle(c, r == ncclSuccess ? ncclSuccess : ncclInProgress,
                                                                    "ncclCommInitRank")
                                                           : nccl_fail(c, r, "ncclCommInitRankConfig");
  if (st != WG_OK) {
    if (c->comm && !c->aborted) N->CommAbort(c->comm);
    release(c);
    return st;
  }
  *out = c;
  return WG_OK;
}

extern "C" wg_status wg_comm_destroy(wg_comm *c) {
  if (!c) return WG_OK;
  NcclApi *N = nccl();
  wg_device_guard guard(c->dev->ordinal);
  if (!c->aborted) {
    cudaStreamSynchronize(c->stream);
    N->CommDestroy(c->comm);
  }
  release(c);
  return WG_OK;
}

extern "C" wg_status wg_comm_abort(wg_comm *c) {
  if (!c) return WG_OK;
  if (!c->aborted) {
    nccl()->CommAbort(c->comm);
    c->aborted = true;
  }
  return WG_OK;
}

extern "C" wg_status wg_comm_rank(const wg_comm *c, int *rank, int *nranks) {
  if (!c || !rank || !nranks) return wg_fail(WG_ERR_INVALID_ARGUMENT, "invalid argument");
  *rank = c->rank;
  *nranks = c->nranks;
  return WG_OK;
}

extern "C" wg_status wg_comm_wait(wg_comm *c) {
  if (!c || c->aborted) return wg_fail(WG_ERR_INVALID_ARGUMENT, "communicator is NULL or aborted");
  wg_device_guard guard(c->dev->ordinal);
  return wait_event(c, c->done, "sharded GEMM");
}

extern "C" wg_status wg_sgemm_sharded(wg_comm *c, int transA, int transB, int64_t m_local, int64_t n, int64_t k,
                                      float alpha, const float *A, int64_t lda, float *B, int64_t ldb, int root,
                                      float beta, float *C, int64_t ldc, int64_t panel_cols) {
  return sharded<float>(c, transA, transB, m_local, n, k, alpha, A, lda, B, ldb, root, beta, C, ldc, panel_cols);
}

extern "C" wg_status wg_dgemm_sharded(wg_comm *c, int transA, int transB, int64_t m_local, int64_t n, int64_t k,
                                      double alpha, const double *A, int64_t lda, double *B, int64_t ldb, int root,
                                      double beta, double *C, int64_t ldc, int64_t panel_cols) {
  return sharded<double>(c, transA, transB, m_local, n, k, alpha, A, lda, B, ldb, root, beta, C, ldc, panel_cols);
}

extern "C" wg_status wg_sgemm_gather_rows(wg_comm *c, const float *C_local, int64_t m_local, int64_t n, int64_t ldc,
                                          int root, float *C_full, int64_t ldc_full, const int64_t *row_offsets) {
  return gather<float>(c, C_local, m_local, n, ldc, root, C_full, ldc_full, row_offsets);
}

extern "C" wg_status wg_dgemm_gather_rows(wg_comm *c, const double *C_local, int64_t m_local, int64_t n,
                                          int64_t ldc, int root, double *C_full, int64_t ldc_full,
                                          const int64_t *row_offsets) {
  return gather<double>(c, C_local, m_local, n, ldc, root, C_full, ldc_full, row_offsets);
}
