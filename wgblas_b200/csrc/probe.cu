// Roofline probes: FP32 FFMA, FP64 DFMA and DMMA peak rates and HBM bandwidth,
// measured with CUDA events on the device handle's stream.
//
// The FMA probes follow the idea of the reference's benchmarks/roofline/wgblas/fma.js:1-72
// (independent multiply-add chains per thread, enough threads to fill every
// SM, a long loop so the issue rate is all that is measured); the bandwidth
// probes stream a buffer much larger than L2 through 16-byte loads and stores.
#include "internal.h"
#include "tcgen05.cuh"

namespace {

constexpr int CHAINS = 8;

__device__ __forceinline__ float fma_t(float a, float b, float c) { return __fmaf_rn(a, b, c); }
__device__ __forceinline__ double fma_t(double a, double b, double c) { return __fma_rn(a, b, c); }

template <typename T>
__global__ void __launch_bounds__(256) fma_probe_kernel(T x, T y, int iters, T *sink) {
  T a[CHAINS];
#pragma unroll
  for (int c = 0; c < CHAINS; c++) a[c] = T(threadIdx.x + c) * T(1e-3);
  for (int i = 0; i < iters; i++) {
#pragma unroll
    for (int c = 0; c < CHAINS; c++) a[c] = fma_t(a[c], x, y);
  }
  T s = T(0);
#pragma unroll
  for (int c = 0; c < CHAINS; c++) s += a[c];
  if (s == T(-12345.678)) sink[threadIdx.x] = s;  // never true; keeps the chains live
}

// Independent chains of FP64 tensor-core MMAs (mma.sync m16n8k8 f64) per warp.
__global__ void __launch_bounds__(256) dmma_probe_kernel(double x, int iters, double *sink) {
  constexpr int CH = 4;
  double acc[CH][4];
  double a[4], b[2];
#pragma unroll
  for (int v = 0; v < 4; v++) a[v] = x * (threadIdx.x + v);
  b[0] = x;
  b[1] = 1.0 - x;
#pragma unroll
  for (int c = 0; c < CH; c++)
#pragma unroll
    for (int v = 0; v < 4; v++) acc[c][v] = 0.0;
  for (int i = 0; i < iters; i++) {
#pragma unroll
    for (int c = 0; c < CH; c++)
      asm volatile(
          "mma.sync.aligned.m16n8k8.row.col.f64.f64.f64.f64 "
          "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
          : "+d"(acc[c][0]), "+d"(acc[c][1]), "+d"(acc[c][2]), "+d"(acc[c][3])
          : "d"(a[0]), "d"(a[1]), "d"(a[2]), "d"(a[3]), "d"(b[0]), "d"(b[1]));
  }
  double s = 0.0;
#pragma unroll
  for (int c = 0; c < CH; c++)
#pragma unroll
    for (int v = 0; v < 4; v++) s += acc[c][v];
  if (s == -12345.678) sink[threadIdx.x] = s;
}

wg_status dmma_probe(wg_device *d, double *tflops) {
  const int blocks = d->sm_count * 4, threads = 256, iters = 1 << 12;
  double *sink = nullptr;
  WG_CUDA(cudaMallocAsync((void **)&sink, threads * sizeof(double), d->stream));
  cudaEvent_t e0, e1;
  WG_CUDA(cudaEventCreate(&e0));
  WG_CUDA(cudaEventCreate(&e1));
  float best = 1e30f;
  for (int rep = 0; rep < 4; rep++) {
    cudaEventRecord(e0, d->stream);
    dmma_probe_kernel<<<blocks, threads, 0, d->stream>>>(1e-3, iters, sink);
    cudaEventRecord(e1, d->stream);
    WG_CUDA(cudaEventSynchronize(e1));
    float ms = 0;
    cudaEventElapsedTime(&ms, e0, e1);
    if (rep > 0 && ms < best) best = ms;
  }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  cudaFreeAsync(sink, d->stream);
  WG_CUDA(cudaStreamSynchronize(d->stream));
  // 4 chains x 16x8x8 MACs per warp per iteration
  const double flops = 2.0 * 16 * 8 * 8 * 4.0 * (double)iters * blocks * (threads / 32);
  *tflops = flops / (best * 1e-3) / 1e12;
  return WG_OK;
}

__global__ void copy_probe_kernel(const float4 *__restrict__ src, float4 *__restrict__ dst, size_t n) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    dst[i] = src[i];
}

// Read-only stream: the store is guarded by a condition the (zeroed) data never
// meets, so nothing is written, but the loads cannot be dropped.
__global__ void read_probe_kernel(const float4 *__restrict__ src, float4 *__restrict__ sink, size_t n) {
  float acc = 0.0f;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const float4 v = src[i];
    acc += (v.x + v.y) + (v.z + v.w);
  }
  if (acc == 1e30f) sink[0] = make_float4(acc, acc, acc, acc);
}

// In-place read-modify-write over one buffer (the sscal shape).
__global__ void scale_probe_kernel(float4 *__restrict__ buf, size_t n) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    float4 v = buf[i];
    v.x *= 1.0000001f;
    v.y *= 1.0000001f;
    v.z *= 1.0000001f;
    v.w *= 1.0000001f;
    buf[i] = v;
  }
}

template <typename T>
wg_status fma_probe(wg_device *d, double *tflops) {
  const int blocks = d->sm_count * 8, threads = 256, iters = 1 << 14;
  T *sink = nullptr;
  WG_CUDA(cudaMallocAsync((void **)&sink, threads * sizeof(T), d->stream));
  cudaEvent_t e0, e1;
  WG_CUDA(cudaEventCreate(&e0));
  WG_CUDA(cudaEventCreate(&e1));
  float best = 1e30f;
  for (int rep = 0; rep < 4; rep++) {
    cudaEventRecord(e0, d->stream);
    fma_probe_kernel<T><<<blocks, threads, 0, d->stream>>>(T(0.999999), T(1e-7), iters, sink);
    cudaEventRecord(e1, d->stream);
    WG_CUDA(cudaEventSynchronize(e1));
    float ms = 0;
    cudaEventElapsedTime(&ms, e0, e1);
    if (rep > 0 && ms < best) best = ms;  // the first launch warms clocks and caches
  }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  cudaFreeAsync(sink, d->stream);
  WG_CUDA(cudaStreamSynchronize(d->stream));
  const double flops = 2.0 * CHAINS * (double)iters * blocks * threads;
  *tflops = flops / (best * 1e-3) / 1e12;
  return WG_OK;
}

// Streams 2 GiB (far above the 126 MB L2) through 16-byte accesses in one of
// three patterns, as the reference's benchmarks/roofline/wgblas/bandwidth.js:1-19
// does, since no single pattern is fastest everywhere: a copy (read + write of
// 2 GiB each), a read-only pass, or an in-place read-modify-write. GB/s counts
// the bytes read plus the bytes written; best of three timed passes after a
// warm-up pass.
wg_status stream_probe(wg_device *d, int kind, double *gbs) {
  const size_t bytes = (size_t)1 << 31;
  const size_t n = bytes / sizeof(float4);
  float4 *src = nullptr, *dst = nullptr;
  WG_CUDA(cudaMallocAsync((void **)&src, bytes, d->stream));
  cudaError_t e = kind == WG_PROBE_HBM_COPY ? cudaMallocAsync((void **)&dst, bytes, d->stream)
                                            : cudaMallocAsync((void **)&dst, sizeof(float4), d->stream);
  if (e != cudaSuccess) {
    cudaFreeAsync(src, d->stream);
    return wg_fail(WG_ERR_OUT_OF_MEMORY, "bandwidth probe allocation failed: %s", cudaGetErrorString(e));
  }
  WG_CUDA(cudaMemsetAsync(src, 0, bytes, d->stream));
  cudaEvent_t e0, e1;
  WG_CUDA(cudaEventCreate(&e0));
  WG_CUDA(cudaEventCreate(&e1));
  float best = 1e30f;
  const unsigned blocks = (unsigned)d->sm_count * 16;
  for (int rep = 0; rep < 4; rep++) {
    cudaEventRecord(e0, d->stream);
    if (kind == WG_PROBE_HBM_COPY)
      copy_probe_kernel<<<blocks, 512, 0, d->stream>>>(src, dst, n);
    else if (kind == WG_PROBE_HBM_READ)
      read_probe_kernel<<<blocks, 512, 0, d->stream>>>(src, dst, n);
    else
      scale_probe_kernel<<<blocks, 512, 0, d->stream>>>(src, n);
    cudaEventRecord(e1, d->stream);
    WG_CUDA(cudaEventSynchronize(e1));
    float ms = 0;
    cudaEventElapsedTime(&ms, e0, e1);
    if (rep > 0 && ms < best) best = ms;
  }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  cudaFreeAsync(src, d->stream);
  cudaFreeAsync(dst, d->stream);
  WG_CUDA(cudaStreamSynchronize(d->stream));
  const double moved = kind == WG_PROBE_HBM_READ ? (double)bytes : 2.0 * (double)bytes;
  *gbs = moved / (best * 1e-3) / 1e9;
  return WG_OK;
}

// One thread waits, with the tensor-core kernels' clock-bounded mbarrier wait,
// on a barrier no thread or copy ever completes; when the budget runs out it
// records the timeout in the device error word and returns.
__global__ void bounded_wait_selftest(unsigned *dwords, long long budget) {
  __shared__ uint64_t bar;
  if (threadIdx.x != 0) return;
  wgtc::mbar_init(&bar, 1);
  wgtc::fence_barrier_init();
  if (!wgtc::mbar_wait_bounded(&bar, 0, budget)) atomicOr(dwords + WG_DW_ERROR, WG_DERR_SELFTEST);
}

}  // namespace

extern "C" wg_status wg_selftest_bounded_wait(wg_device *d, unsigned budget_us) {
  if (!d) return wg_fail(WG_ERR_INVALID_ARGUMENT, "device is NULL");
  if (budget_us == 0 || budget_us > 1000000) return wg_fail(WG_ERR_INVALID_ARGUMENT, "budget_us must be in (0, 1e6]");
  wg_device_guard guard(d->ordinal);
  int khz = 0;
  WG_CUDA(cudaDeviceGetAttribute(&khz, cudaDevAttrClockRate, d->ordinal));
  const long long budget = (long long)budget_us * (khz > 0 ? khz / 1000 : 2000);
  wg_launch_scope scope(d, "selftest_bounded_wait");
  bounded_wait_selftest<<<1, 32, 0, d->stream>>>(d->dwords, budget);
  WG_CUDA(cudaGetLastError());
  return WG_OK;
}

extern "C" wg_status wg_probe_peak(wg_device *d, int kind, double *value) {
  if (!d || !value) return wg_fail(WG_ERR_INVALID_ARGUMENT, "invalid argument");
  wg_device_guard guard(d->ordinal);
  switch (kind) {
    case WG_PROBE_FP32_FMA: return fma_probe<float>(d, value);
    case WG_PROBE_FP64_FMA: return fma_probe<double>(d, value);
    case WG_PROBE_HBM_COPY:
    case WG_PROBE_HBM_READ:
    case WG_PROBE_HBM_SCALE: return stream_probe(d, kind, value);
    case WG_PROBE_FP64_DMMA: return dmma_probe(d, value);
    default: return wg_fail(WG_ERR_INVALID_ARGUMENT, "unknown probe %d", kind);
  }
}
