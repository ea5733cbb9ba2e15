// Device handles, buffers, page-locked host memory, errors and seeded inputs of
// the wgblas-b200 C ABI (include/wgblas.h).
//
// What this replaces in the reference:
//   src/init.mjs:31-143        init / cleanup / gpuName  -> wg_device_*
//   src/util/buffer.mjs:58-78  uploadBuffer               -> wg_buffer_upload*
//   src/util/result.mjs:18-29  mapAsync readback          -> wg_buffer_download*
//   src/random/random.mjs:4-26 seeded generators          -> wg_random_*
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>
#include <set>
#include <tuple>

#include "internal.h"

static thread_local char g_last_error[1024] = "";

wg_status wg_fail(wg_status st, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof g_last_error, fmt, ap);
  va_end(ap);
  return st;
}

extern "C" const char *wg_last_error(void) { return g_last_error; }

cudaError_t wg_kernel_smem_raw(const void *fn, size_t bytes, bool max_carveout) {
  static std::mutex mu;
  static std::set<std::tuple<const void *, int, size_t, bool>> done;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const auto key = std::make_tuple(fn, dev, bytes, max_carveout);
  std::lock_guard<std::mutex> lock(mu);
  if (done.count(key)) return cudaSuccess;
  e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e == cudaSuccess && max_carveout)
    e = cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
  if (e == cudaSuccess) done.insert(key);
  return e;
}
extern "C" int wg_abi_version(void) { return WG_ABI_VERSION; }

// ---------------------------------------------------------------------------
// devices
// ---------------------------------------------------------------------------

extern "C" wg_status wg_device_count(int *count) {
  if (!count) return wg_fail(WG_ERR_INVALID_ARGUMENT, "count is NULL");
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver) {
    cudaGetLastError();
    n = 0;
  } else if (e != cudaSuccess) {
    return wg_fail(WG_ERR_CUDA, "cudaGetDeviceCount failed: %s", cudaGetErrorString(e));
  }
  *count = n;
  return WG_OK;
}

extern "C" wg_status wg_device_open(int ordinal, unsigned flags, wg_device **out) {
  if (!out) return wg_fail(WG_ERR_INVALID_ARGUMENT, "out is NULL");
  *out = nullptr;
  int n = 0;
  wg_status st = wg_device_count(&n);
  if (st != WG_OK) return st;
  if (n == 0) return wg_fail(WG_ERR_NO_DEVICE, "no CUDA device is visible");
  if (ordinal < 0 || ordinal >= n)
    return wg_fail(WG_ERR_NO_DEVICE, "device ordinal %d out of range (%d visible)", ordinal, n);
  cudaDeviceProp prop;
  WG_CUDA(cudaGetDeviceProperties(&prop, ordinal));
  wg_device_guard guard(ordinal);
  wg_device *d = new (std::nothrow) wg_device();
  if (!d) return wg_fail(WG_ERR_OUT_OF_MEMORY, "host allocation failed");
  d->ordinal = ordinal;
  d->flags = flags;
  d->sm_count = prop.multiProcessorCount;
  d->cc_major = prop.major;
  d->cc_minor = prop.minor;
  d->total_mem = prop.totalGlobalMem;
  snprintf(d->name, sizeof d->name, "%s", prop.name);
  cudaError_t e = cudaStreamCreateWithFlags(&d->own_stream, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaEventCreate(&d->ev_start);
  if (e == cudaSuccess) e = cudaEventCreate(&d->ev_stop);
  if (e == cudaSuccess) e = cudaMalloc(&d->dwords, WG_DW_COUNT * sizeof(unsigned));
  if (e == cudaSuccess) e = cudaMemsetAsync(d->dwords, 0, WG_DW_COUNT * sizeof(unsigned), d->own_stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(d->own_stream);
  if (e != cudaSuccess) {
    if (d->dwords) cudaFree(d->dwords);
    if (d->ev_stop) cudaEventDestroy(d->ev_stop);
    if (d->ev_start) cudaEventDestroy(d->ev_start);
    if (d->own_stream) cudaStreamDestroy(d->own_stream);
    delete d;
    return wg_fail(e == cudaErrorMemoryAllocation ? WG_ERR_OUT_OF_MEMORY : WG_ERR_CUDA,
                   "opening device %d failed: %s", ordinal, cudaGetErrorString(e));
  }
  d->stream = d->own_stream;
  d->sgemm_path = WG_SGEMM_AUTO;
  d->dgemm_path = WG_DGEMM_AUTO;
  d->strsm_path = WG_STRSM_AUTO;
  wg_noalloc_reserve(ordinal);  // wg_sgemm_noalloc's fixed scratch is reserved now, not at its first call
  *out = d;
  return WG_OK;
}

extern "C" wg_status wg_device_close(wg_device *d) {
  if (!d) return WG_OK;  // unknown or released handles are a no-op (src/init.mjs:120-122)
  wg_device_guard guard(d->ordinal);
  cudaStreamSynchronize(d->stream);
  if (d->ws) cudaFree(d->ws);
  if (d->flow_flags) cudaFree(d->flow_flags);
  if (d->dwords) cudaFree(d->dwords);
  cudaEventDestroy(d->ev_start);
  cudaEventDestroy(d->ev_stop);
  for (auto &p : d->pending) {
    cudaEventDestroy(p.e0);
    cudaEventDestroy(p.e1);
  }
  for (cudaEvent_t e : d->event_pool) cudaEventDestroy(e);
  if (d->h2d) cudaStreamDestroy(d->h2d);
  if (d->d2h) cudaStreamDestroy(d->d2h);
  if (d->staging) cudaMemPoolDestroy(d->staging);
  if (d->side) {
    cudaStreamSynchronize(d->side);
    cudaStreamDestroy(d->side);
  }
  for (cudaEvent_t e : d->tc_ev)
    if (e) cudaEventDestroy(e);
  cudaStreamDestroy(d->own_stream);
  delete d;
  return WG_OK;
}

extern "C" wg_status wg_device_name(const wg_device *d, char *buf, size_t len) {
  if (!d || !buf || len == 0) return wg_fail(WG_ERR_INVALID_ARGUMENT, "invalid argument");
  snprintf(buf, len, "%s", d->name);
  return WG_OK;
}

extern "C" wg_status wg_device_props_get(const wg_device *d, wg_device_props *p) {
  if (!d || !p) return wg_fail(WG_ERR_INVALID_ARGUMENT, "invalid argument");
  p->ordinal = d->ordinal;
  p->sm_count = d->sm_count;
  p->cc_major = d->cc_major;
  p->cc_minor = d->cc_minor;
  p->total_mem = d->total_mem;
  p->flags = d->flags;
  return WG_OK;
}

extern "C" wg_status wg_device_stream(const wg_device *d, void **stream) {
  if (!d || !stream) return wg_fail(WG_ERR_INVALID_ARGUMENT, "invalid argument");
  *stream = (void *)d->stream;
  return WG_OK;
}

extern "C" wg_status wg_device_set_stream(wg_device *d, void *stream) {
  if (!d) return wg_fail(WG_ERR_INVALID_ARGUMENT, "device is NULL");
  d->stream = stream ? (cudaStream_t)stream : d->own_stream;
  return WG_OK;
}

extern "C" wg_status wg_device_sync(wg_device *d) {
  if (!d) return wg_fail(WG_ERR_INVALID_ARGUMENT, "device is NULL");
  wg_device_guard guard(d->ordinal);
  WG_CUDA(cudaStreamSynchronize(d->stream));
  return WG_OK;
}

extern "C" wg_status wg_device_check(wg_device *d) {
  if (!d) return wg_fail(WG_ERR_INVALID_ARGUMENT, "device is NULL");
  wg_device_guard guard(d->ordinal);
  unsigned word = 0;
  WG_CUDA(cudaMemcpyAsync(&word, d->dwords + WG_DW_ERROR, sizeof word, cudaMemcpyDeviceToHost, d->stream));
  WG_CUDA(cudaStreamSynchronize(d->stream));
  if (word) {
    WG_CUDA(cudaMemsetAsync(d->dwords + WG_DW_ERROR, 0, sizeof(unsigned), d->stream));
    WG_CUDA(cudaStreamSynchronize(d->stream));
    return wg_fail(WG_ERR_KERNEL_TIMEOUT,
                   "a kernel's bounded wait gave up (device error word 0x%x); its output "
                   "is incomplete", word);
  }
  return WG_OK;
}

extern "C" wg_status wg_device_sgemm_stats(wg_device *d, wg_sgemm_stats *s) {
  if (!d || !s) return wg_fail(WG_ERR_INVALID_ARGUMENT, "invalid argument");
  wg_device_guard guard(d->ordinal);
  unsigned fb = 0;
  WG_CUDA(cudaMemcpyAsync(&fb, d->dwords + WG_DW_FALLBACKS, sizeof fb, cudaMemcpyDeviceToHost, d->stream));
  WG_CUDA(cudaStreamSynchronize(d->stream));
  *s = d->stats;
  s->fallbacks = fb;
  return WG_OK;
}

// ---- per-kernel profiling -------------------------------------------------

static cudaEvent_t pool_event(wg_device *d) {
  if (!d->event_pool.empty()) {
    cudaEvent_t e = d->event_pool.back();
    d->event_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  cudaEventCreate(&e);
  return e;
}

wg_launch_scope::wg_launch_scope(wg_device *dev, const char *family, cudaStream_t stream)
    : d(dev), s(stream ? stream : dev->stream), slot(-1) {
  d->launches++;
  if (!d->profiling) return;
  int f = -1;
  for (size_t i = 0; i < d->families.size(); i++)
    if (d->families[i] == family) f = (int)i;
  if (f < 0) {
    d->families.push_back(family);
    d->fam_launches.push_back(0);
    d->fam_ms.push_back(0.0);
    f = (int)d->families.size() - 1;
  }
  wg_device::pending_t p{f, pool_event(d), pool_event(d)};
  if (!p.e0 || !p.e1) return;
  cudaEventRecord(p.e0, s);
  d->pending.push_back(p);
  slot = (int)d->pending.size() - 1;
}

wg_launch_scope::~wg_launch_scope() {
  if (slot >= 0) cudaEventRecord(d->pending[slot].e1, s);
}

extern "C" wg_status wg_device_set_profiling(wg_device *d, int on) {
  if (!d) return wg_fail(WG_ERR_INVALID_ARGUMENT, "device is NULL");
  d->profiling = on != 0;
  return WG_OK;
}

extern "C" wg_status wg_device_profile_read(wg_device *d, wg_kernel_profile *out, int max, int *count) {
  if (!d || !count || (max > 0 && !out)) return wg_fail(WG_ERR_INVALID_ARGUMENT, "invalid argument");
  wg_device_guard guard(d->ordinal);
  WG_CUDA(cudaStreamSynchronize(d->stream));
  if (d->side) WG_CUDA(cudaStreamSynchronize(d->side));
  for (auto &p : d->pending) {
    float ms = 0.0f;
    if (cudaEventElapsedTime(&ms, p.e0, p.e1) == cudaSuccess) {
      d->fam_ms[p.family] += ms;
      d->fam_launches[p.family]++;
    }
    d->event_pool.push_back(p.e0);
    d->event_pool.push_back(p.e1);
  }
  d->pending.clear();
  int n = 0;
  for (size_t i = 0; i < d->families.size() && n < max; i++) {
    if (!d->fam_launches[i]) continue;
    snprintf(out[n].name, sizeof out[n].name, "%s", d->families[i].c_str());
    out[n].launches = d->fam_launches[i];
    out[n].total_ms = d->fam_ms[i];
    n++;
  }
  for (size_t i = 0; i < d->families.size(); i++) {
    d->fam_launches[i] = 0;
    d->fam_ms[i] = 0.0;
  }
  *count = n;
  return WG_OK;
}

extern "C" wg_status wg_device_kernel_launches(const wg_device *d, uint64_t *launches) {
  if (!d || !launches) return wg_fail(WG_ERR_INVALID_ARGUMENT, "invalid argument");
  *launches = d->launches;
  return WG_OK;
}

extern "C" wg_status wg_device_set_dgemm_path(wg_device *d, int path) {
  if (!d) return wg_fail(WG_ERR_INVALID_ARGUMENT, "device is NULL");
  if (path != WG_DGEMM_AUTO && path != WG_DGEMM_SIMT && path != WG_DGEMM_DMMA)
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "unknown dgemm path %d", path);
  d->dgemm_path = path;
  return WG_OK;
}

extern "C" wg_status wg_device_set_strsm_path(wg_device *d, int path) {
  if (!d) return wg_fail(WG_ERR_INVALID_ARGUMENT, "device is NULL");
  if (path != WG_STRSM_AUTO && path != WG_STRSM_RECURSIVE && path != WG_STRSM_FLOW)
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "unknown strsm path %d", path);
  d->strsm_path = path;
  return WG_OK;
}

extern "C" wg_status wg_device_set_sgemm_path(wg_device *d, int path) {
  if (!d) return wg_fail(WG_ERR_INVALID_ARGUMENT, "device is NULL");
  if (path < WG_SGEMM_AUTO || path > WG_SGEMM_SIMT_SMALL)
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "unknown sgemm path %d", path);
  d->sgemm_path = path;
  d->fused_bn = path == WG_SGEMM_TF32X3_FUSED_BN256 ? 256
              : path == WG_SGEMM_TF32X3_FUSED_BN128 ? 128
              : path == WG_SGEMM_TF32X3_FUSED_BN64 ? 64 : 0;
  return WG_OK;
}

wg_status wg_workspace(wg_device *d, size_t bytes, void **ptr) {
  if (bytes > d->ws_bytes) {
    if (d->ws) {
      // The old scratch may still be read by queued kernels: free it in stream order.
      WG_CUDA(cudaStreamSynchronize(d->stream));
      WG_CUDA(cudaFree(d->ws));
      d->ws = nullptr;
      d->ws_bytes = 0;
    }
    size_t want = (bytes + ((size_t)1 << 21) - 1) & ~(((size_t)1 << 21) - 1);
    WG_CUDA(cudaMalloc(&d->ws, want));
    d->ws_bytes = want;
  }
  *ptr = d->ws;
  return WG_OK;
}

// ---------------------------------------------------------------------------
// buffers
// ---------------------------------------------------------------------------

extern "C" wg_status wg_buffer_alloc(wg_device *d, size_t bytes, wg_buffer **out) {
  if (!d || !out) return wg_fail(WG_ERR_INVALID_ARGUMENT, "invalid argument");
  *out = nullptr;
  wg_device_guard guard(d->ordinal);
  wg_buffer *b = (wg_buffer *)calloc(1, sizeof(wg_buffer));
  if (!b) return wg_fail(WG_ERR_OUT_OF_MEMORY, "host allocation failed");
  b->dev = d;
  b->bytes = bytes;
  if (bytes) {
    cudaError_t e = cudaMalloc(&b->ptr, bytes);
    if (e != cudaSuccess) {
      free(b);
      return wg_fail(e == cudaErrorMemoryAllocation ? WG_ERR_OUT_OF_MEMORY : WG_ERR_CUDA,
                     "cudaMalloc(%zu) failed: %s", bytes, cudaGetErrorString(e));
    }
  }
  *out = b;
  return WG_OK;
}

wg_status wg_staging_pool(wg_device *d) {
  if (d->staging) return WG_OK;
  cudaMemPoolProps props = {};
  props.allocType = cudaMemAllocationTypePinned;
  props.location.type = cudaMemLocationTypeDevice;
  props.location.id = d->ordinal;
  cudaMemPool_t pool = nullptr;
  WG_CUDA(cudaMemPoolCreate(&pool, &props));
  uint64_t keep = UINT64_MAX;  // release threshold: keep what has been mapped
  cudaError_t e = cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
  if (e != cudaSuccess) {
    cudaMemPoolDestroy(pool);
    return wg_fail(WG_ERR_CUDA, "cudaMemPoolSetAttribute failed: %s", cudaGetErrorString(e));
  }
  d->staging = pool;
  return WG_OK;
}

extern "C" wg_status wg_buffer_alloc_async(wg_device *d, size_t bytes, wg_buffer **out) {
  if (!d || !out) return wg_fail(WG_ERR_INVALID_ARGUMENT, "invalid argument");
  *out = nullptr;
  wg_device_guard guard(d->ordinal);
  wg_status st = wg_staging_pool(d);
  if (st != WG_OK) return st;
  wg_buffer *b = (wg_buffer *)calloc(1, sizeof(wg_buffer));
  if (!b) return wg_fail(WG_ERR_OUT_OF_MEMORY, "host allocation failed");
  b->dev = d;
  b->bytes = bytes;
  b->pooled = 1;
  if (bytes) {
    cudaError_t e = cudaMallocFromPoolAsync(&b->ptr, bytes, d->staging, d->stream);
    if (e != cudaSuccess) {
      free(b);
      return wg_fail(e == cudaErrorMemoryAllocation ? WG_ERR_OUT_OF_MEMORY : WG_ERR_CUDA,
                     "cudaMallocFromPoolAsync(%zu) failed: %s", bytes, cudaGetErrorString(e));
    }
  }
  *out = b;
  return WG_OK;
}

extern "C" wg_status wg_buffer_free(wg_buffer *b) {
  if (!b) return WG_OK;
  wg_device_guard guard(b->dev->ordinal);
  if (b->pooled) {
    // Returned to the pool in stream order, after the work queued so far.
    if (b->ptr) cudaFreeAsync(b->ptr, b->dev->stream);
  } else {
    // Work queued on the owning stream may still read the buffer.
    cudaStreamSynchronize(b->dev->stream);
    if (b->ptr) cudaFree(b->ptr);
  }
  free(b);
  return WG_OK;
}

extern "C" wg_status wg_buffer_size(const wg_buffer *b, size_t *bytes) {
  if (!b || !bytes) return wg_fail(WG_ERR_INVALID_ARGUMENT, "invalid argument");
  *bytes = b->bytes;
  return WG_OK;
}

extern "C" wg_status wg_buffer_device_ptr(const wg_buffer *b, void **ptr) {
  if (!b || !ptr) return wg_fail(WG_ERR_INVALID_ARGUMENT, "invalid argument");
  *ptr = b->ptr;
  return WG_OK;
}

static bool span_ok(size_t off, size_t len, size_t size) { return off <= size && len <= size - off; }

extern "C" wg_status wg_buffer_upload(wg_buffer *b, size_t off, const void *host, size_t bytes) {
  if (!b || (!host && bytes)) return wg_fail(WG_ERR_INVALID_ARGUMENT, "invalid argument");
  if (!span_ok(off, bytes, b->bytes))
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "upload of %zu bytes at %zu exceeds the %zu-byte buffer",
                   bytes, off, b->bytes);
  if (!bytes) return WG_OK;
  wg_device_guard guard(b->dev->ordinal);
  WG_CUDA(cudaMemcpyAsync((char *)b->ptr + off, host, bytes, cudaMemcpyHostToDevice, b->dev->stream));
  // The host array may be released as soon as this returns.
  WG_CUDA(cudaStreamSynchronize(b->dev->stream));
  return WG_OK;
}

extern "C" wg_status wg_buffer_download(const wg_buffer *b, size_t off, void *host, size_t bytes) {
  if (!b || (!host && bytes)) return wg_fail(WG_ERR_INVALID_ARGUMENT, "invalid argument");
  if (!span_ok(off, bytes, b->bytes))
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "download of %zu bytes at %zu exceeds the %zu-byte buffer",
                   bytes, off, b->bytes);
  if (!bytes) return WG_OK;
  wg_device_guard guard(b->dev->ordinal);
  WG_CUDA(cudaMemcpyAsync(host, (const char *)b->ptr + off, bytes, cudaMemcpyDeviceToHost, b->dev->stream));
  WG_CUDA(cudaStreamSynchronize(b->dev->stream));
  return WG_OK;
}

static bool span2d_ok(size_t off, size_t pitch, size_t width, size_t rows, size_t size) {
  if (rows == 0 || width == 0) return true;
  if (width > pitch) return false;
  size_t last = (rows - 1) * pitch;
  if (rows > 1 && last / (rows - 1) != pitch) return false;
  return span_ok(off, last + width, size);
}

extern "C" wg_status wg_buffer_upload_2d(wg_buffer *b, size_t off, size_t dpitch, const void *host,
                                         size_t spitch, size_t width, size_t rows) {
  if (!b || (!host && width && rows) || (rows > 1 && spitch < width))
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "invalid argument");
  if (!span2d_ok(off, dpitch, width, rows, b->bytes))
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "strided upload exceeds the %zu-byte buffer", b->bytes);
  if (!width || !rows) return WG_OK;
  wg_device_guard guard(b->dev->ordinal);
  WG_CUDA(cudaMemcpy2DAsync((char *)b->ptr + off, dpitch, host, spitch ? spitch : width, width, rows,
                            cudaMemcpyHostToDevice, b->dev->stream));
  WG_CUDA(cudaStreamSynchronize(b->dev->stream));
  return WG_OK;
}

extern "C" wg_status wg_buffer_download_2d(const wg_buffer *b, size_t off, size_t spitch, void *host,
                                           size_t dpitch, size_t width, size_t rows) {
  if (!b || (!host && width && rows) || (rows > 1 && dpitch < width))
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "invalid argument");
  if (!span2d_ok(off, spitch, width, rows, b->bytes))
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "strided download exceeds the %zu-byte buffer", b->bytes);
  if (!width || !rows) return WG_OK;
  wg_device_guard guard(b->dev->ordinal);
  WG_CUDA(cudaMemcpy2DAsync(host, dpitch ? dpitch : width, (const char *)b->ptr + off, spitch, width, rows,
                            cudaMemcpyDeviceToHost, b->dev->stream));
  WG_CUDA(cudaStreamSynchronize(b->dev->stream));
  return WG_OK;
}

extern "C" wg_status wg_host_alloc(size_t bytes, void **ptr) {
  if (!ptr) return wg_fail(WG_ERR_INVALID_ARGUMENT, "ptr is NULL");
  *ptr = nullptr;
  WG_CUDA(cudaHostAlloc(ptr, bytes ? bytes : 1, cudaHostAllocPortable));
  return WG_OK;
}

extern "C" wg_status wg_host_free(void *ptr) {
  if (ptr) WG_CUDA(cudaFreeHost(ptr));
  return WG_OK;
}

// ---------------------------------------------------------------------------
// seeded inputs — src/random/random.mjs:4-26
// ---------------------------------------------------------------------------

// One mulberry32 draw in [0, 1) (random.mjs:4-12). The JS computes in int32 with
// Math.imul and `>>>`; both are the same as uint32 arithmetic mod 2^32.
static inline double mulberry32(uint32_t &a) {
  a += 0x6d2b79f5u;
  uint32_t t = (a ^ (a >> 15)) * (1u | a);
  t = (t + (t ^ (t >> 7)) * (61u | t)) ^ t;
  return (double)(t ^ (t >> 14)) / 4294967296.0;
}

extern "C" void wg_random_f32(float *out, int64_t n, double low, double high, uint32_t seed) {
  uint32_t s = seed;
  for (int64_t i = 0; i < n; i++) out[i] = (float)(low + mulberry32(s) * (high - low));
}

extern "C" void wg_random_f64(double *out, int64_t n, double low, double high, uint32_t seed) {
  uint32_t s = seed;
  for (int64_t i = 0; i < n; i++) out[i] = low + mulberry32(s) * (high - low);
}

// Box-Muller: r = sqrt(-2 ln(1 - u1)), z0 = r cos(2 pi u2), z1 = r sin(2 pi u2).
template <typename T>
static void normal_fill(T *out, int64_t n, uint32_t seed) {
  uint32_t s = seed;
  const double two_pi = 6.283185307179586476925286766559;
  for (int64_t i = 0; i < n; i += 2) {
    double u1 = mulberry32(s);
    double u2 = mulberry32(s);
    double r = std::sqrt(-2.0 * std::log(1.0 - u1));
    out[i] = (T)(r * std::cos(two_pi * u2));
    if (i + 1 < n) out[i + 1] = (T)(r * std::sin(two_pi * u2));
  }
}

extern "C" void wg_random_normal_f32(float *out, int64_t n, uint32_t seed) { normal_fill(out, n, seed); }
extern "C" void wg_random_normal_f64(double *out, int64_t n, uint32_t seed) { normal_fill(out, n, seed); }
