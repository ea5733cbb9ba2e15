// sgemm for callers that cannot allocate device memory.
//
// Some programs must not have a library call cudaMalloc on their behalf: a
// host application whose own allocator reserves all of the device's memory up
// front and hands out nothing else, or a real-time loop where an allocation
// (which can synchronise the device) would stall. wg_sgemm_noalloc serves them.
// It runs the 3xTF32 tensor-core kernels with their split-operand scratch in a
// fixed array compiled into this library, instead of the grow-only workspace
// the other entry points allocate. The caller still passes A, B and C as
// device pointers.
//
// The array (g_noalloc_scratch, WG_NOALLOC_SCRATCH_BYTES = 64 MiB) is a
// file-scope __device__ variable. Under CUDA's lazy module loading (the
// default since CUDA 12.2) the runtime reserves it on a GPU only when the code
// object holding it is first used there, which would make the first call the
// one that allocates. So wg_device_open looks the array's address up
// (cudaGetSymbolAddress, with the device current) and caches it per device:
// the array is reserved when the handle is opened and stays reserved until
// the process exits. Open the handle before the application's own allocator
// takes the device's memory. Host code cannot use the array's name as a
// device address; every call passes the cached address to the kernels. If
// the lookup failed at open, the first call retries it (and then should come
// before any stream capture).
//
// Every call on a device shares the one array, and the array keeps the last
// call's contents. Each call rewrites every element it reads (the pack pass
// writes the whole padded operand region, zeros included), so nothing needs
// clearing. Calls whose work overlaps on the GPU — on different streams or
// device handles of the same GPU — race on the array: order them on one
// stream.
#include <cstdio>
#include <mutex>

#include "internal.h"

namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[WG_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mutex;
void *g_scratch_addr[kMaxDevices];  // device address of g_noalloc_scratch, per ordinal

// Looks up (once per device, with that device current) the address of the array.
wg_status scratch_address(int ordinal, void **out) {
  if (ordinal < 0 || ordinal >= kMaxDevices)
    return wg_fail(WG_ERR_NOT_SUPPORTED, "device ordinal %d is beyond this library's table", ordinal);
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (!g_scratch_addr[ordinal]) {
    wg_device_guard guard(ordinal);
    void *p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return wg_fail(WG_ERR_CUDA, "cudaGetSymbolAddress of the no-allocation scratch failed on device %d: %s",
                     ordinal, cudaGetErrorString(e));
    g_scratch_addr[ordinal] = p;
  }
  *out = g_scratch_addr[ordinal];
  return WG_OK;
}

}  // namespace

void wg_noalloc_reserve(int ordinal) {
  char saved[1024];
  snprintf(saved, sizeof saved, "%s", wg_last_error());
  void *p = nullptr;
  if (scratch_address(ordinal, &p) != WG_OK) wg_fail(WG_OK, "%s", saved);  // retried by the first call
}

extern "C" wg_status wg_sgemm_noalloc(wg_device *d, int transA, int transB, int64_t m, int64_t n, int64_t k,
                                      float alpha, const float *A, int64_t lda, const float *B, int64_t ldb,
                                      float beta, float *C, int64_t ldc) {
  if (!d) return wg_fail(WG_ERR_INVALID_ARGUMENT, "device is NULL");
  if ((transA != 0 && transA != 1) || (transB != 0 && transB != 1))
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "transA and transB must be 0 (no-transpose) or 1 (transpose)");
  if (m < 0 || n < 0 || k < 0) return wg_fail(WG_ERR_INVALID_ARGUMENT, "m, n, and k must be non-negative.");
  if (lda < (transA ? k : m) || ldb < (transB ? n : k) || ldc < m || lda <= 0 || ldb <= 0 || ldc <= 0)
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "a leading dimension is below the rows of its matrix as stored");
  if (m == 0 || n == 0) return WG_OK;
  if (!C || (k > 0 && alpha != 0.0f && (!A || !B)))
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "operand pointer is NULL");
  if (d->cc_major != 10)
    return wg_fail(WG_ERR_NOT_SUPPORTED, "device %d is not an sm_100 device", d->ordinal);
  wg_device_guard guard(d->ordinal);
  if (alpha == 0.0f || k == 0) {  // C = alpha*0 + beta*C needs no scratch
    wg_launch_scope scope(d, "scale");
    WG_CUDA(wg_launch_scale<float>(d->stream, m, n, alpha, beta, C, ldc));
    return WG_OK;
  }
  if (!wg_tf32x3_supported(d, m, n, k))
    return wg_fail(WG_ERR_NOT_SUPPORTED,
                   "wg_sgemm_noalloc runs the 3xTF32 kernel, which needs k >= 8 (got m=%lld n=%lld k=%lld)",
                   (long long)m, (long long)n, (long long)k);
  const size_t need = wg_tf32x3_workspace_bytes(m, n, k);
  if (need > WG_NOALLOC_SCRATCH_BYTES)
    return wg_fail(WG_ERR_INVALID_ARGUMENT,
                   "m=%lld n=%lld k=%lld needs %zu bytes of split-operand scratch; wg_sgemm_noalloc holds at "
                   "most %zu bytes (2*(round_up(m,128) + round_up(n,256))*round_up(k,32)*4 must fit)",
                   (long long)m, (long long)n, (long long)k, need, (size_t)WG_NOALLOC_SCRATCH_BYTES);
  void *ws = nullptr;
  wg_status st = scratch_address(d->ordinal, &ws);
  if (st != WG_OK) return st;
  // Whole-tile scheduling: the fixed array holds the split operands only.
  return wg_sgemm_tf32x3(d, transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, ws, need);
}
