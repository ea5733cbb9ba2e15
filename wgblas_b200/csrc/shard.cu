// Multi-GPU sgemm / dgemm: C sharded by row blocks across ranks, the shared
// operand B sent from `root` to every other rank over NVLink, one process (or
// device handle) per GPU.
//
// The reference has no multi-GPU exchange at all (several independent
// GPUDevices, src/init.mjs:14-29); this is the sharding the north star asks
// for. Rank r owns rows [off_r, off_r + m_r) of C and of op(A), resident on its
// GPU (scattered once). Each call sends root's B in column panels into every
// other rank's landing buffer; the GEMM of panel j waits only for panel j, so
// the transfer of panel j+1 overlaps the math of panel j.
//
// Transport: on one node with the ranks on distinct GPUs, a copy-engine chain
// (root -> root+1 -> ...): each rank's DMA engines push 16 MiB chunks into its
// successor's landing buffer (an IPC mapping) and raise the successor's
// arrival counter with a stream memory write, and a one-warp kernel with a
// clock-bounded spin waits for each chunk. No SM moves data, so the GEMMs keep
// every SM. Otherwise ncclBroadcast. Every compute kernel reads only its own
// GPU's memory (no peer loads, no TMA multicast).
//
// NCCL (libnccl.so.2) is opened at run time, so the library loads on machines
// without it and shares the copy a host framework already loaded. It carries
// the setup exchanges, the planning all-reduce, the fallback broadcast and the
// gather. The communicator is created non-blocking and every wait, on NCCL or
// on a neighbour's chunk, is bounded by the communicator's timeout, after which
// it is aborted and WG_ERR_NCCL is returned: a rank that never joins or dies
// surfaces as an error instead of a hang.
#include <cuda.h>
#include <dlfcn.h>
#include <cstdlib>
#include <nccl.h>

#include <algorithm>
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
  ncclResult_t (*AllGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
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
    // WGBLAS_NCCL_LIBRARY names a specific NCCL (the Python layer points it at the
    // copy bundled with torch, so that a later `import torch` binds to the same
    // library instead of failing on an older system NCCL that took its soname).
    // Local symbol scope: nothing of NCCL is exported to libraries loaded later.
    void *h = nullptr;
    const char *path = getenv("WGBLAS_NCCL_LIBRARY");
    if (path && *path) h = dlopen(path, RTLD_NOW | RTLD_LOCAL);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
    if (!h) return;
#define LOAD(field, sym) api.field = reinterpret_cast<decltype(api.field)>(dlsym(h, sym))
    LOAD(GetUniqueId, "ncclGetUniqueId");
    LOAD(CommInitRankConfig, "ncclCommInitRankConfig");
    LOAD(CommDestroy, "ncclCommDestroy");
    LOAD(CommAbort, "ncclCommAbort");
    LOAD(CommGetAsyncError, "ncclCommGetAsyncError");
    LOAD(Broadcast, "ncclBroadcast");
    LOAD(AllReduce, "ncclAllReduce");
    LOAD(AllGather, "ncclAllGather");
    LOAD(Send, "ncclSend");
    LOAD(Recv, "ncclRecv");
    LOAD(GroupStart, "ncclGroupStart");
    LOAD(GroupEnd, "ncclGroupEnd");
    LOAD(GetErrorString, "ncclGetErrorString");
#undef LOAD
    api.ok = api.GetUniqueId && api.CommInitRankConfig && api.CommDestroy && api.CommAbort &&
             api.CommGetAsyncError && api.Broadcast && api.AllReduce && api.AllGather && api.Send && api.Recv && api.GroupStart && api.GroupEnd &&
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
  // Root's B reaches the other ranks in their landing buffer (`land`, same
  // leading dimension as B). With the copy-engine chain (ranks on distinct GPUs
  // of one node) rank r copies each chunk into rank r+1's landing buffer over
  // NVLink with the DMA engines and raises rank r+1's arrival counter, so no SM
  // runs the transfer; otherwise ncclBroadcast fills it.
  struct Chain {
    bool on;
    unsigned long long *flags;       // local: [0] chunks landed, [1] successor ready (its call count)
    unsigned long long *next_flags;  // rank+1's flags (IPC mapping)
    unsigned long long *prev_flags;  // rank-1's flags (IPC mapping)
    unsigned *err;                   // set by a wait that ran out of time
    char *land, *next_land;          // landing buffers (root's B arrives here): this rank's, rank+1's
    size_t land_bytes;
    cudaStream_t s;                  // the chain's stream
    std::vector<cudaEvent_t> ev;     // chunk landed (recorded on s)
    cudaEvent_t end_s;
    unsigned long long seq, calls;   // chunks and calls so far (the same on every rank)
    long long budget;                // SM clock cycles a wait may spin
  } ce;
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

void release_chain(wg_comm::Chain &ce) {
  if (ce.next_land) cudaIpcCloseMemHandle(ce.next_land);
  if (ce.next_flags) cudaIpcCloseMemHandle(ce.next_flags);
  if (ce.prev_flags && ce.prev_flags != ce.next_flags) cudaIpcCloseMemHandle(ce.prev_flags);
  if (ce.land) cudaFree(ce.land);
  if (ce.flags) cudaFree(ce.flags);
  if (ce.err) cudaFree(ce.err);
  for (cudaEvent_t e : ce.ev) cudaEventDestroy(e);
  if (ce.end_s) cudaEventDestroy(ce.end_s);
  if (ce.s) cudaStreamDestroy(ce.s);
  ce = wg_comm::Chain{};
}

// ---- copy-engine chain broadcast ------------------------------------------

typedef CUresult (*WriteValue64Fn)(CUstream, CUdeviceptr, cuuint64_t, unsigned int);

WriteValue64Fn write_value64() {
  static WriteValue64Fn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuStreamWriteValue64", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<WriteValue64Fn>(p);
  });
  return fn;
}

// One thread waits, for at most `budget` SM clock cycles, until *flag reaches
// `target`. The flag lives in this GPU's memory and is raised by the
// predecessor rank's copy stream over NVLink (after the chunk it announces has
// landed, or when its landing buffer is free); a wait that runs out sets *err
// and returns, so a rank that never arrives becomes an error, not a hang.
__global__ void chain_wait(const volatile unsigned long long *flag, unsigned long long target, long long budget,
                           unsigned *err) {
  if (threadIdx.x != 0) return;
  const long long t0 = clock64();
  while (*flag < target) {
    if (clock64() - t0 > budget) {
      atomicOr(err, 1u);
      return;
    }
    __nanosleep(256);
  }
}

// Gathers `bytes` of host data from every rank (rank order) through NCCL; every
// wait is bounded by the communicator's timeout.
wg_status allgather_host(wg_comm *c, const void *mine, void *all, size_t bytes) {
  char *dev = nullptr, *host = nullptr;
  const size_t total = bytes * (size_t)c->nranks;
  WG_CUDA(cudaHostAlloc((void **)&host, total, cudaHostAllocDefault));
  cudaError_t e = cudaMalloc((void **)&dev, bytes + total);
  wg_status st = WG_OK;
  if (e == cudaSuccess) e = cudaMemcpyAsync(dev, mine, bytes, cudaMemcpyHostToDevice, c->stream);
  if (e != cudaSuccess) st = wg_fail(WG_ERR_CUDA, "all-gather staging failed: %s", cudaGetErrorString(e));
  if (st == WG_OK)
    st = settle(c, nccl()->AllGather(dev, dev + bytes, bytes, ncclUint8, c->comm, c->stream), "ncclAllGather");
  if (st == WG_OK) {
    e = cudaMemcpyAsync(host, dev + bytes, total, cudaMemcpyDeviceToHost, c->stream);
    if (e == cudaSuccess) e = cudaEventRecord(c->agreed, c->stream);
    st = e == cudaSuccess ? wait_event(c, c->agreed, "ncclAllGather")
                          : wg_fail(WG_ERR_CUDA, "all-gather read-back failed: %s", cudaGetErrorString(e));
  }
  if (st == WG_OK) memcpy(all, host, total);
  if (st == WG_OK || !c->aborted) {
    cudaStreamSynchronize(c->stream);
    if (dev) cudaFree(dev);
  }
  cudaFreeHost(host);
  return st;
}

struct ChainInfo {
  cudaIpcMemHandle_t flags;
  unsigned char uuid[16];
  int ok;
};

// Sets up the chain (collective): flag words shared by IPC with both
// neighbours. It is used only when every rank can: distinct GPUs, IPC and
// stream memory operations available; otherwise B goes out with ncclBroadcast.
wg_status chain_setup(wg_comm *c) {
  wg_comm::Chain &ce = c->ce;
  ce = wg_comm::Chain{};
  if (c->nranks < 2) return WG_OK;
  ChainInfo mine;
  memset(&mine, 0, sizeof mine);
  cudaDeviceProp prop;
  bool ok = write_value64() != nullptr && cudaGetDeviceProperties(&prop, c->dev->ordinal) == cudaSuccess;
  if (ok) memcpy(mine.uuid, &prop.uuid, sizeof mine.uuid);
  ok = ok && cudaMalloc((void **)&ce.flags, 256) == cudaSuccess && cudaMemset(ce.flags, 0, 256) == cudaSuccess &&
       cudaMalloc((void **)&ce.err, sizeof(unsigned)) == cudaSuccess &&
       cudaMemset(ce.err, 0, sizeof(unsigned)) == cudaSuccess &&
       cudaIpcGetMemHandle(&mine.flags, ce.flags) == cudaSuccess &&
       cudaStreamCreateWithFlags(&ce.s, cudaStreamNonBlocking) == cudaSuccess &&
       cudaEventCreateWithFlags(&ce.end_s, cudaEventDisableTiming) == cudaSuccess &&
       cudaDeviceSynchronize() == cudaSuccess;
  cudaGetLastError();
  mine.ok = ok ? 1 : 0;
  std::vector<ChainInfo> all(c->nranks);
  wg_status st = allgather_host(c, &mine, all.data(), sizeof(ChainInfo));
  if (st != WG_OK) return st;
  bool all_ok = true;
  for (int r = 0; r < c->nranks; r++) {
    all_ok = all_ok && all[r].ok;
    for (int q = 0; q < r; q++) all_ok = all_ok && memcmp(all[r].uuid, all[q].uuid, 16) != 0;
  }
  const int next = (c->rank + 1) % c->nranks, prev = (c->rank + c->nranks - 1) % c->nranks;
  int opened = 0;
  if (all_ok) {
    opened = cudaIpcOpenMemHandle((void **)&ce.next_flags, all[next].flags, cudaIpcMemLazyEnablePeerAccess) ==
             cudaSuccess;
    if (opened && prev == next) ce.prev_flags = ce.next_flags;
    else if (opened)
      opened = cudaIpcOpenMemHandle((void **)&ce.prev_flags, all[prev].flags, cudaIpcMemLazyEnablePeerAccess) ==
               cudaSuccess;
    cudaGetLastError();
  }
  // Every rank must take the same path.
  std::vector<int> opened_all(c->nranks);
  st = allgather_host(c, &opened, opened_all.data(), sizeof(int));
  if (st != WG_OK) return st;
  bool on = all_ok;
  for (int v : opened_all) on = on && v;
  if (!on) {
    release_chain(ce);
    return WG_OK;
  }
  int khz = 0;
  cudaDeviceGetAttribute(&khz, cudaDevAttrClockRate, c->dev->ordinal);
  ce.budget = (long long)c->timeout_ms * (khz > 0 ? khz : 2000000);
  ce.on = true;
  return WG_OK;
}

// Grows this rank's landing buffer to `bytes` (the ranks call it with the same
// size). With the chain it is collective: nothing may be in flight into or out
// of the old buffers on any rank, every rank closes its mapping of its
// successor's buffer before any rank frees the one it exported (an all-gather
// is the barrier between), and the new buffers are exchanged by IPC.
wg_status grow_landing(wg_comm *c, size_t bytes) {
  wg_comm::Chain &ce = c->ce;
  if (bytes <= ce.land_bytes) return WG_OK;
  if (ce.s) WG_CUDA(cudaStreamSynchronize(ce.s));
  WG_CUDA(cudaStreamSynchronize(c->stream));
  WG_CUDA(cudaStreamSynchronize(c->dev->stream));  // GEMMs reading the old buffer
  if (c->dev->side) WG_CUDA(cudaStreamSynchronize(c->dev->side));
  wg_status st = WG_OK;
  if (ce.on) {
    if (ce.next_land) cudaIpcCloseMemHandle(ce.next_land);
    ce.next_land = nullptr;
    int dummy = 0;
    std::vector<int> sink(c->nranks);
    st = allgather_host(c, &dummy, sink.data(), sizeof(int));
    if (st != WG_OK) return st;
  }
  if (ce.land) cudaFree(ce.land);
  ce.land = nullptr;
  ce.land_bytes = 0;
  cudaError_t e = cudaMalloc((void **)&ce.land, bytes);
  if (ce.on) {
    cudaIpcMemHandle_t mine;
    memset(&mine, 0, sizeof mine);
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&mine, ce.land);
    std::vector<cudaIpcMemHandle_t> all(c->nranks);
    st = allgather_host(c, &mine, all.data(), sizeof mine);
    if (st != WG_OK) return st;
    if (e == cudaSuccess)
      e = cudaIpcOpenMemHandle((void **)&ce.next_land, all[(c->rank + 1) % c->nranks],
                               cudaIpcMemLazyEnablePeerAccess);
  }
  if (e != cudaSuccess)
    return wg_fail(e == cudaErrorMemoryAllocation ? WG_ERR_OUT_OF_MEMORY : WG_ERR_CUDA,
                   "landing buffer of %zu bytes for root's B: %s", bytes, cudaGetErrorString(e));
  ce.land_bytes = bytes;
  return WG_OK;
}

cudaEvent_t chain_event(wg_comm::Chain &ce, size_t i) {
  while (ce.ev.size() <= i) {
    cudaEvent_t e = nullptr;
    cudaEventCreateWithFlags(&e, cudaEventDisableTiming);
    ce.ev.push_back(e);
  }
  return ce.ev[i];
}

// One column range of the stored B (rows_s x cols_s) moved as a unit.
struct Chunk {
  int64_t col0, cols;
};

// Queues this rank's part of the chain for one call: B (stored rows_s x
// cols_s, leading dimension ldb, on `root`) travels root -> root+1 -> ... in
// `chunks`; each other rank receives it in its landing buffer (the same
// leading dimension) and forwards it. chunk_ev[i] fires when chunk i is
// present on this rank (in B on the root, in the landing buffer elsewhere).
wg_status chain_broadcast(wg_comm *c, int root, const char *B, int64_t ldb, int64_t rows_s, size_t elt,
                          const std::vector<Chunk> &chunks, cudaEvent_t entry) {
  wg_comm::Chain &ce = c->ce;
  WriteValue64Fn wv = write_value64();
  const int P = c->nranks, me = c->rank;
  const int next = (me + 1) % P;
  const bool is_root = me == root, forward = next != root;
  const unsigned long long call = ce.calls + 1;
  const size_t col_bytes = (size_t)rows_s * elt, pitch = (size_t)ldb * elt;
  WG_CUDA(cudaStreamWaitEvent(ce.s, entry, 0));
  // This rank's landing buffer is free (everything before this call has read
  // it): tell the predecessor, and wait for the same word from the successor.
  if (!is_root && wv((CUstream)ce.s, (CUdeviceptr)(ce.prev_flags + 1), call, 0) != CUDA_SUCCESS)
    return wg_fail(WG_ERR_CUDA, "cuStreamWriteValue64 failed");
  if (forward) {
    chain_wait<<<1, 32, 0, ce.s>>>(ce.flags + 1, call, ce.budget, ce.err);
    WG_CUDA(cudaGetLastError());
  }
  for (size_t i = 0; i < chunks.size(); i++) {
    const Chunk &k = chunks[i];
    const size_t off = (size_t)k.col0 * pitch;
    if (!is_root) {
      chain_wait<<<1, 32, 0, ce.s>>>(ce.flags, ce.seq + i + 1, ce.budget, ce.err);
      WG_CUDA(cudaGetLastError());
    }
    WG_CUDA(cudaEventRecord(chain_event(ce, i), ce.s));
    if (forward) {
      const char *src = is_root ? B + off : ce.land + off;
      WG_CUDA(cudaMemcpy2DAsync(ce.next_land + off, pitch, src, pitch, col_bytes, (size_t)k.cols,
                                cudaMemcpyDeviceToDevice, ce.s));
      if (wv((CUstream)ce.s, (CUdeviceptr)ce.next_flags, ce.seq + i + 1, 0) != CUDA_SUCCESS)
        return wg_fail(WG_ERR_CUDA, "cuStreamWriteValue64 failed");
    }
  }
  WG_CUDA(cudaEventRecord(ce.end_s, ce.s));
  ce.seq += chunks.size();
  ce.calls = call;
  return WG_OK;
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
  if (c->ce.s) cudaStreamSynchronize(c->ce.s);
  release_chain(c->ce);
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
  if (n == 0 || k == 0) {
    // Nothing to broadcast; each rank scales its own block (k == 0) or has nothing to do.
    if (m_local && n) return wg_gemm_enqueue<T>(c->dev, transA, transB, m_local, n, k, alpha, A, lda, B, ldb, beta,
                                                C, ldc);
    return WG_OK;
  }
  if (c->rank == root && !B) return wg_fail(WG_ERR_INVALID_ARGUMENT, "B is NULL on the root");
  NcclApi *N = nccl();
  wg_device *d = c->dev;
  wg_device_guard guard(d->ordinal);
  // Panel widths, the same on every rank: one panel for a transposed B (its
  // columns are not contiguous), the caller's width when given, planned widths
  // for an sgemm the 3xTF32 kernel can take, else one panel.
  std::vector<int64_t> widths;
  const bool auto_plan = std::is_same<T, float>::value && !transB && panel <= 0 && k >= 64;
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
  // Root's B reaches the other ranks in their landing buffer (leading dimension
  // ldb): by the copy-engine chain when the ranks set one up, else by
  // ncclBroadcast. The chain moves the stored B (rows_s x cols_s) in chunks of
  // at most 16 MiB cut inside the panels; a panel is ready when its last chunk
  // is. A chunk reaches the last of P ranks after P-1 hops, so small chunks keep
  // the first panel's wait short (7 hops of 16 MiB at about 700 GB/s: 0.17 ms).
  constexpr int64_t CHUNK_BYTES = (int64_t)16 << 20;
  const bool chain = c->ce.on;
  const int64_t rows_s = transB ? n : k, cols_s = transB ? k : n;
  if (c->nranks > 1) {
    wg_status st = grow_landing(c, (size_t)ldb * (size_t)cols_s * sizeof(T));
    if (st != WG_OK) return st;
  }
  std::vector<Chunk> chunks;
  std::vector<size_t> panel_last;
  if (chain) {
    const int64_t per = std::max<int64_t>(1, CHUNK_BYTES / (rows_s * (int64_t)sizeof(T)));
    int64_t c0 = 0;
    for (size_t j = 0; j < widths.size(); j++) {
      const int64_t w = transB ? cols_s : widths[j];
      const int64_t nc = (w + per - 1) / per;
      for (int64_t i = 0; i < nc; i++) {
        const int64_t a = c0 + w * i / nc, b = c0 + w * (i + 1) / nc;
        chunks.push_back(Chunk{a, b - a});
      }
      panel_last.push_back(chunks.size() - 1);
      c0 += w;
    }
  }
  // Root's B must be ready, and every earlier reader of the landing buffer done, before the transfer.
  WG_CUDA(cudaEventRecord(c->entry, d->stream));
  if (chain) {
    wg_status st = chain_broadcast(c, root, reinterpret_cast<const char *>(B), ldb, rows_s, sizeof(T), chunks,
                                   c->entry);
    if (st != WG_OK) return st;
  } else {
    WG_CUDA(cudaStreamWaitEvent(c->stream, c->entry, 0));
  }
  // Where op(B) is read on this rank: B on the root, the landing buffer elsewhere.
  const bool from_land = c->nranks > 1 && c->rank != root;
  T *Bsrc = from_land ? reinterpret_cast<T *>(c->ce.land) : B;
  // On the tensor cores the panels form one product: op(A) is split once, and
  // each arriving panel's split overlaps the previous panel's MMA.
  wg_tc_product prod{};
  wg_status st = WG_OK;
  if (tc)
    st = wg_tc_product_begin(&prod, d, transA, transB, m_local, k, (float)alpha, (const float *)A, lda, (float)beta,
                             widths.data(), widths.size(), nullptr, (const float *)Bsrc, ldb);
  int64_t j0 = 0;
  for (size_t j = 0; st == WG_OK && j < widths.size(); j++) {
    const int64_t cols = widths[j];
    // Column panel of a column-major k x n B (transB = 0), or all of the n x k B.
    T *bp = Bsrc + (transB ? 0 : j0 * ldb);
    cudaEvent_t ev;
    cudaError_t e = cudaSuccess;
    if (chain) {
      ev = chain_event(c->ce, panel_last[j]);
    } else {
      const size_t count = transB ? (size_t)((k - 1) * ldb + n) : (size_t)((cols - 1) * ldb + k);
      const T *send = c->rank == root ? bp : nullptr;
      st = settle(c, N->Broadcast(send, bp, count, nccl_type<T>(), root, c->comm, c->stream), "ncclBroadcast");
      if (st != WG_OK) break;
      ev = panel_event(c, j);
      e = cudaEventRecord(ev, c->stream);
    }
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
  // The chain's copies out of this rank's buffers are done before the call is.
  if (chain) cudaStreamWaitEvent(d->stream, c->ce.end_s, 0);
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
  if (st == WG_OK) st = chain_setup(c);
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
    if (c->ce.on) {
      // Close the mappings of the neighbours' memory on every rank before any
      // rank frees what it exported.
      cudaStreamSynchronize(c->ce.s);
      wg_comm::Chain &ce = c->ce;
      if (ce.next_land) cudaIpcCloseMemHandle(ce.next_land);
      if (ce.next_flags) cudaIpcCloseMemHandle(ce.next_flags);
      if (ce.prev_flags && ce.prev_flags != ce.next_flags) cudaIpcCloseMemHandle(ce.prev_flags);
      ce.next_land = nullptr;
      ce.next_flags = ce.prev_flags = nullptr;
      int dummy = 0;
      std::vector<int> sink(c->nranks);
      allgather_host(c, &dummy, sink.data(), sizeof(int));
    }
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
  wg_status st = wait_event(c, c->done, "sharded GEMM");
  if (st != WG_OK || !c->ce.on) return st;
  unsigned err = 0;
  WG_CUDA(cudaMemcpy(&err, c->ce.err, sizeof err, cudaMemcpyDeviceToHost));
  if (err) {
    nccl()->CommAbort(c->comm);
    c->aborted = true;
    return wg_fail(WG_ERR_NCCL, "broadcast chain: rank %d waited %d ms for its neighbour's data and gave up; "
                   "communicator aborted", c->rank, c->timeout_ms);
  }
  return WG_OK;
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
