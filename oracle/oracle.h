/*
 * CPU oracle for the wgblas level-3 GEMM path (sgemm / dgemm).
 *
 * TEST INFRASTRUCTURE ONLY. Nothing in the product library links, loads or
 * calls this code; it is imported by tests/, by __graft_entry__.smoke() as the
 * checker, and by bench.py's cpu_baseline / --impl reference leg as the timed
 * CPU restatement of the reference's arithmetic.
 *
 * Every routine works in the column-major BLAS frame:
 *   C[i + j*ldc] := alpha * sum_p op(A)(i,p) * op(B)(p,j) + beta * C[i + j*ldc]
 *   op(A)(i,p) = transA ? A[p + i*lda] : A[i + p*lda]
 *   op(B)(p,j) = transB ? B[j + p*ldb] : B[p + j*ldb]
 * The reference kernels run in a row-major frame after a layout swap
 * (src/sgemm/sgemm.mjs:151-167); each output element is still one sequential
 * dot product over p = 0..k-1 followed by the same epilogue, so the per-element
 * arithmetic restated here does not depend on the frame.
 *
 * Parity pins: tests/golden/ holds the reference's own edge-case inputs with
 * exact expected outputs, the double-double lane cases of
 * tests/shaders/src/test.dekker.js and the split/merge cases of
 * tests/utils/test.f64.js; tests/test_oracle.py checks this file against them.
 */
#ifndef WGBLAS_ORACLE_H
#define WGBLAS_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- seeded inputs: src/random/random.mjs:4-26 --------------------------- */
/* mulberry32 state and one draw in [0, 1), as in random.mjs:4-12. */
double or_mulberry32_next(uint32_t *state);
/* randomFloat32Array(n, low, high, seed): low + next()*(high-low), stored as f32. */
void or_random_f32(float *out, int64_t n, double low, double high, uint32_t seed);
/* randomFloat64Array(n, low, high, seed). */
void or_random_f64(double *out, int64_t n, double low, double high, uint32_t seed);
/* Standard normal draws (Box-Muller over mulberry32; the reference has none). */
void or_random_normal_f32(float *out, int64_t n, uint32_t seed);
void or_random_normal_f64(double *out, int64_t n, uint32_t seed);

/* ---- sgemm restatement: src/shaders/sgemm_large.wgsl:112-308 ------------- */
/* variant 0: every product and sum rounded separately (no contraction).
 * variant 1: acc = fmaf(a, b, acc) and the beta term fused, as an FMA-contracting
 * shader compiler emits it. Writes C in place. nthreads <= 0 means all cores. */
void or_sgemm(int variant, int transA, int transB, int64_t m, int64_t n, int64_t k,
              float alpha, const float *A, int64_t lda, const float *B, int64_t ldb,
              float beta, float *C, int64_t ldc, int nthreads);
/* fp64-accumulated truth of the same product. out (ldo) gets alpha*AB + beta*C in
 * double; absab (ldo, may be NULL) gets sum_p |op(A)(i,p)|*|op(B)(p,j)|. */
void or_sgemm_truth(int transA, int transB, int64_t m, int64_t n, int64_t k,
                    float alpha, const float *A, int64_t lda, const float *B, int64_t ldb,
                    float beta, const float *C, int64_t ldc,
                    double *out, double *absab, int64_t ldo, int nthreads);

/* ---- dgemm restatements --------------------------------------------------- */
/* The reference's double-double dgemm (src/dgemm/dgemm.mjs:177-304): host split,
 * dgemm_small.wgsl per-element arithmetic, exact merge. C in place. Includes the
 * quick return (alpha==0 or k==0) and beta==1. variant 0 rounds every operation
 * as written; variant 1 fuses ddMul's unprotected cross-term product-sum
 * (batch.wgsl:106), the one place a contracting compiler can fuse. */
void or_dgemm_dd(int variant, int transA, int transB, int64_t m, int64_t n, int64_t k,
                 double alpha, const double *A, int64_t lda, const double *B, int64_t ldb,
                 double beta, double *C, int64_t ldc, int nthreads);
/* Native fp64: acc = fma(a, b, acc) in increasing p, then the same epilogue with the
 * beta term fused. The CUDA DFMA kernel is expected to match it bit for bit. */
void or_dgemm_fma(int transA, int transB, int64_t m, int64_t n, int64_t k,
                  double alpha, const double *A, int64_t lda, const double *B, int64_t ldb,
                  double beta, double *C, int64_t ldc, int nthreads);
/* long-double-accumulated truth; out/absab as in or_sgemm_truth. */
void or_dgemm_truth(int transA, int transB, int64_t m, int64_t n, int64_t k,
                    double alpha, const double *A, int64_t lda, const double *B, int64_t ldb,
                    double beta, const double *C, int64_t ldc,
                    double *out, double *absab, int64_t ldo, int nthreads);

/* ---- double-double primitives (src/shaders/f64/utils/ add, multiply, batch) ------------- */
void or_dd_two_sum(float a, float b, float *hi, float *lo);          /* add.wgsl:88-98 (twoSumProtected) */
void or_dd_fast_two_sum(float a, float b, float *hi, float *lo);     /* add.wgsl:100-110 */
void or_dd_two_prod_bit(float a, float b, float *hi, float *lo);     /* multiply.wgsl:32-45 */
void or_dd_add(float ahi, float alo, float bhi, float blo, float *hi, float *lo); /* add.wgsl:112-116 */
void or_dd_mul(float ahi, float alo, float bhi, float blo, float *hi, float *lo); /* batch.wgsl:103-109 */
/* src/util/f64.mjs:33-43 and :80-91 */
void or_dd_split(const double *x, float *hi, float *lo, int64_t n);
void or_dd_merge(const float *hi, const float *lo, double *out, int64_t n);
void or_dd_merge_exact(const float *hi, const float *lo, const double *before,
                       double *out, int64_t n);

/* Number of worker threads or_* routines use for nthreads <= 0. */
int or_default_threads(void);

#ifdef __cplusplus
}
#endif
#endif
