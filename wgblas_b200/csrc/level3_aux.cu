// The operand passes that ssymm/dsymm and strmm/dtrmm put in front of a GEMM,
// as the reference does (src/ssymm/ssymm.mjs:26-28 with symmetrize.wgsl,
// src/strmm/strmm.mjs with triangularize.wgsl): a dense copy of the symmetric
// or triangular operand, after which the product is a plain sgemm / dgemm on
// this library's kernels. Also the device-to-device block copy the in-place
// strmm result needs.
//
// Both passes are HBM-bound copies (one read, one write per element of the
// n x n result) over 32 x 32 tiles staged in shared memory: a tile whose values
// come from the mirrored triangle (symmetrize) or from the transpose (trmm's
// transposed operand) is read as the mirror tile, coalesced along its columns,
// and written transposed, coalesced along the output's columns. Only the
// referenced triangle of A is ever read. At 4096 x 4096 symmetrize takes 56 us
// and triangularize 52 us (62 and 58 elementwise, with the mirrored reads
// strided), about 2.3 TB/s of read plus write.
#include "internal.h"

namespace {

constexpr int TT = 32;  // tile edge; 256 threads = 32 x 8
// Tiles per block step, all loaded before any is stored. Four (16 loads per
// thread in flight) measured no faster than one at 4096 (60 against 58 us for
// symmetrize): the pass is not bound by loads in flight.
constexpr int TQ = 1;

// out(i, j) = A(i, j) where (i, j) is in the stored triangle (lower: i >= j,
// upper: i <= j, column-major frame), A(j, i) elsewhere.
template <typename T>
__global__ void __launch_bounds__(256) symmetrize_kernel(int64_t n, int lower, const T *__restrict__ A, int64_t lda,
                                                         T *__restrict__ out, int64_t ldo) {
  __shared__ T S[TQ][TT][TT + 1];  // S[q][c][r] = A(si*TT + r, sj*TT + c) of the q-th tile
  const int tx = threadIdx.x % TT, ty = threadIdx.x / TT;
  const int64_t tiles = (n + TT - 1) / TT, total = tiles * tiles;
  for (int64_t t0 = (int64_t)blockIdx.x * TQ; t0 < total; t0 += (int64_t)gridDim.x * TQ) {
    __syncthreads();  // the previous tiles' reads of S are done
#pragma unroll
    for (int q = 0; q < TQ; q++) {  // every load of the TQ tiles before any store
      const int64_t t = t0 + q;
      if (t >= total) break;
      const int64_t bi = t % tiles, bj = t / tiles;  // output tile: rows bi*TT.., columns bj*TT..
      const bool diag = bi == bj, stored_tile = lower ? bi > bj : bi < bj;
      // The tile holding these values: this one (stored side, or the diagonal), else its mirror.
      const int64_t si = (stored_tile || diag) ? bi : bj, sj = (stored_tile || diag) ? bj : bi;
#pragma unroll
      for (int c = ty; c < TT; c += 8) {
        const int64_t gi = si * TT + tx, gj = sj * TT + c;
        const bool in = gi < n && gj < n && (!diag || (lower ? gi >= gj : gi <= gj));
        S[q][c][tx] = in ? A[gi + gj * lda] : T(0);
      }
    }
    __syncthreads();
#pragma unroll
    for (int q = 0; q < TQ; q++) {
      const int64_t t = t0 + q;
      if (t >= total) break;
      const int64_t bi = t % tiles, bj = t / tiles;
      const bool diag = bi == bj, stored_tile = lower ? bi > bj : bi < bj;
#pragma unroll
      for (int c = ty; c < TT; c += 8) {
        const int64_t i = bi * TT + tx, j = bj * TT + c;
        if (i >= n || j >= n) continue;
        T v;
        if (diag)
          v = (lower ? i >= j : i <= j) ? S[q][c][tx] : S[q][tx][c];  // A(i, j), or A(j, i) from the same tile
        else
          v = stored_tile ? S[q][c][tx] : S[q][tx][c];
        out[i + j * ldo] = v;
      }
    }
  }
}

// T(i, j) = 1 on the diagonal when `unit` (A's diagonal is not read), A(i, j)
// inside the stored triangle, 0 outside; out = T, or T^T when `trans`.
template <typename T>
__global__ void __launch_bounds__(256) triangularize_kernel(int64_t n, int lower, int unit, int trans,
                                                            const T *__restrict__ A, int64_t lda, T *__restrict__ out,
                                                            int64_t ldo) {
  __shared__ T S[TQ][TT][TT + 1];  // S[q][c][r] = A(si*TT + r, sj*TT + c) of the q-th tile
  const int tx = threadIdx.x % TT, ty = threadIdx.x / TT;
  const int64_t tiles = (n + TT - 1) / TT, total = tiles * tiles;
  for (int64_t t0 = (int64_t)blockIdx.x * TQ; t0 < total; t0 += (int64_t)gridDim.x * TQ) {
    __syncthreads();
#pragma unroll
    for (int q = 0; q < TQ; q++) {  // every load of the TQ tiles before any store
      const int64_t t = t0 + q;
      if (t >= total) break;
      const int64_t br = t % tiles, bc = t / tiles;              // output tile: rows br*TT.., columns bc*TT..
      const int64_t si = trans ? bc : br, sj = trans ? br : bc;  // the tile of T (and of A) they come from
      if (lower ? si < sj : si > sj) continue;                   // wholly outside the triangle: zeros
#pragma unroll
      for (int c = ty; c < TT; c += 8) {
        const int64_t gi = si * TT + tx, gj = sj * TT + c;
        T v = T(0);
        if (gi < n && gj < n) {
          if (gi == gj)
            v = unit ? T(1) : A[gi + gj * lda];
          else if (lower ? gi > gj : gi < gj)
            v = A[gi + gj * lda];
        }
        S[q][c][tx] = v;
      }
    }
    __syncthreads();
#pragma unroll
    for (int q = 0; q < TQ; q++) {
      const int64_t t = t0 + q;
      if (t >= total) break;
      const int64_t br = t % tiles, bc = t / tiles;
      const int64_t si = trans ? bc : br, sj = trans ? br : bc;
      const bool outside = lower ? si < sj : si > sj;
#pragma unroll
      for (int c = ty; c < TT; c += 8) {
        const int64_t r = br * TT + tx, cc = bc * TT + c;
        if (r >= n || cc >= n) continue;
        out[r + cc * ldo] = outside ? T(0) : (trans ? S[q][tx][c] : S[q][c][tx]);
      }
    }
  }
}

unsigned blocks_for(wg_device *d, int64_t n) {
  const int64_t tiles = (n + TT - 1) / TT, want = (tiles * tiles + TQ - 1) / TQ;
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
    symmetrize_kernel<float><<<blocks_for(d, n), 256, 0, d->stream>>>(
        n, lower, static_cast<const float *>(A->ptr) + offA, lda, static_cast<float *>(out->ptr) + offO, ldo);
  else
    symmetrize_kernel<double><<<blocks_for(d, n), 256, 0, d->stream>>>(
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
    triangularize_kernel<float><<<blocks_for(d, n), 256, 0, d->stream>>>(
        n, lower, unit, trans, static_cast<const float *>(A->ptr) + offA, lda, static_cast<float *>(out->ptr) + offO,
        ldo);
  else
    triangularize_kernel<double><<<blocks_for(d, n), 256, 0, d->stream>>>(
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
