// The operand passes that ssymm/dsymm and strmm/dtrmm put in front of a GEMM,
// as the reference does (src/ssymm/ssymm.mjs:26-28 with symmetrize.wgsl,
// src/strmm/strmm.mjs with triangularize.wgsl): a dense copy of the symmetric
// or triangular operand, after which the product is a plain sgemm / dgemm on
// this library's kernels. Also the device-to-device block copy the in-place
// strmm result needs.
//
// Both passes are HBM-bound elementwise copies (one read, one write per element
// of the n x n result; reads of the mirrored triangle are strided but stay in L2
// for the sizes these routines see), grid-stride over column-major output so
// every warp writes 32 consecutive elements of one column.
#include "internal.h"

namespace {

// out(i, j) = A(i, j) where (i, j) is in the stored triangle (lower: i >= j,
// upper: i <= j, column-major frame), A(j, i) elsewhere.
template <typename T>
__global__ void symmetrize_kernel(int64_t n, int lower, const T *__restrict__ A, int64_t lda, T *__restrict__ out,
                                  int64_t ldo) {
  const int64_t total = n * n;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t i = e % n, j = e / n;
    const bool stored = lower ? i >= j : i <= j;
    out[i + j * ldo] = stored ? A[i + j * lda] : A[j + i * lda];
  }
}

// T(i, j) = 1 on the diagonal when `unit` (A's diagonal is not read), A(i, j)
// inside the stored triangle, 0 outside; out = T, or T^T when `trans`.
template <typename T>
__global__ void triangularize_kernel(int64_t n, int lower, int unit, int trans, const T *__restrict__ A, int64_t lda,
                                     T *__restrict__ out, int64_t ldo) {
  const int64_t total = n * n;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = e % n, c = e / n;
    const int64_t i = trans ? c : r, j = trans ? r : c;  // the element of T that lands at out(r, c)
    T v;
    if (i == j)
      v = unit ? T(1) : A[i + j * lda];
    else
      v = (lower ? i > j : i < j) ? A[i + j * lda] : T(0);
    out[r + c * ldo] = v;
  }
}

unsigned blocks_for(wg_device *d, int64_t total) {
  const int64_t want = (total + 255) / 256;
  const int64_t cap = (int64_t)d->sm_count * 16;
  return (unsigned)(want < cap ? (want > 0 ? want : 1) : cap);
}

bool fits_square(const wg_buffer *b, int64_t off, int64_t n, int64_t ld, size_t elt) {
  if (!b || off < 0 || ld < n) return false;
  const int64_t need = off + (n - 1) * ld + n;
  return n == 0 || (size_t)need * elt <= b->bytes;
}

wg_status check_pass(wg_device *d, int elem_bytes, int uplo, int64_t n, const wg_buffer *A, int64_t offA, int64_t lda,
                     const wg_buffer *out, int64_t offO, int64_t ldo) {
  if (!d) return wg_fail(WG_ERR_INVALID_ARGUMENT, "device is NULL");
  if (elem_bytes != 4 && elem_bytes != 8) return wg_fail(WG_ERR_INVALID_ARGUMENT, "elem_bytes must be 4 or 8");
  if (uplo != WG_UPLO_LOWER && uplo != WG_UPLO_UPPER)
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "uplo must be 'lower' or 'upper'.");
  if (n < 0 || lda <= 0 || ldo <= 0) return wg_fail(WG_ERR_INVALID_ARGUMENT, "n must be >= 0, lda and ldo positive");
  if (!fits_square(A, offA, n, lda, (size_t)elem_bytes) || !fits_square(out, offO, n, ldo, (size_t)elem_bytes))
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "a buffer is too small for the n x n matrix and its leading dimension");
  if (A->dev->ordinal != d->ordinal || out->dev->ordinal != d->ordinal)
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "a buffer belongs to another device");
  return WG_OK;
}

}  // namespace

extern "C" wg_status wg_symmetrize(wg_device *d, int elem_bytes, int uplo, int64_t n, const wg_buffer *A, int64_t offA,
                                   int64_t lda, wg_buffer *out, int64_t offO, int64_t ldo) {
  wg_status st = check_pass(d, elem_bytes, uplo, n, A, offA, lda, out, offO, ldo);
  if (st != WG_OK || n == 0) return st;
  wg_device_guard guard(d->ordinal);
  wg_launch_scope scope(d, "symmetrize");
  const int lower = uplo == WG_UPLO_LOWER;
  if (elem_bytes == 4)
    symmetrize_kernel<float><<<blocks_for(d, n * n), 256, 0, d->stream>>>(
        n, lower, static_cast<const float *>(A->ptr) + offA, lda, static_cast<float *>(out->ptr) + offO, ldo);
  else
    symmetrize_kernel<double><<<blocks_for(d, n * n), 256, 0, d->stream>>>(
        n, lower, static_cast<const double *>(A->ptr) + offA, lda, static_cast<double *>(out->ptr) + offO, ldo);
  WG_CUDA(cudaGetLastError());
  return WG_OK;
}

extern "C" wg_status wg_triangularize(wg_device *d, int elem_bytes, int uplo, int trans, int unit, int64_t n,
                                      const wg_buffer *A, int64_t offA, int64_t lda, wg_buffer *out, int64_t offO,
                                      int64_t ldo) {
  wg_status st = check_pass(d, elem_bytes, uplo, n, A, offA, lda, out, offO, ldo);
  if (st != WG_OK || n == 0) return st;
  if ((trans != 0 && trans != 1) || (unit != 0 && unit != 1))
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "trans and unit must be 0 or 1");
  wg_device_guard guard(d->ordinal);
  wg_launch_scope scope(d, "triangularize");
  const int lower = uplo == WG_UPLO_LOWER;
  if (elem_bytes == 4)
    triangularize_kernel<float><<<blocks_for(d, n * n), 256, 0, d->stream>>>(
        n, lower, unit, trans, static_cast<const float *>(A->ptr) + offA, lda, static_cast<float *>(out->ptr) + offO,
        ldo);
  else
    triangularize_kernel<double><<<blocks_for(d, n * n), 256, 0, d->stream>>>(
        n, lower, unit, trans, static_cast<const double *>(A->ptr) + offA, lda,
        static_cast<double *>(out->ptr) + offO, ldo);
  WG_CUDA(cudaGetLastError());
  return WG_OK;
}

extern "C" wg_status wg_buffer_copy_2d(wg_device *d, const wg_buffer *src, size_t src_off, size_t src_pitch,
                                       wg_buffer *dst, size_t dst_off, size_t dst_pitch, size_t width, size_t rows) {
  if (!d || !src || !dst) return wg_fail(WG_ERR_INVALID_ARGUMENT, "device or buffer is NULL");
  if (rows == 0 || width == 0) return WG_OK;
  if (width > src_pitch || width > dst_pitch)
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "the row width exceeds a pitch");
  if (src_off + (rows - 1) * src_pitch + width > src->bytes || dst_off + (rows - 1) * dst_pitch + width > dst->bytes)
    return wg_fail(WG_ERR_INVALID_ARGUMENT, "the block does not fit a buffer");
  wg_device_guard guard(d->ordinal);
  WG_CUDA(cudaMemcpy2DAsync(static_cast<char *>(dst->ptr) + dst_off, dst_pitch,
                            static_cast<const char *>(src->ptr) + src_off, src_pitch, width, rows,
                            cudaMemcpyDeviceToDevice, d->stream));
  return WG_OK;
}
