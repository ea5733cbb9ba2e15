/*
 * CPU oracle for the wgblas GEMM path — TEST INFRASTRUCTURE, never product code.
 * See oracle.h for the frame, the entry points and what pins them.
 *
 * Built with -ffp-contract=off (oracle/Makefile): every float operation written
 * below rounds exactly as written, which is what the reference's "protected"
 * double-double ops enforce on the GPU (src/shaders/f64/utils/add.wgsl:1-15).
 * Fused multiply-adds appear only where fmaf()/fma() is called by name.
 */
#include "oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

/* ------------------------------------------------------------------------- */
/* threads                                                                    */
/* ------------------------------------------------------------------------- */

int or_default_threads(void) {
  long n = sysconf(_SC_NPROCESSORS_ONLN);
  return n > 0 ? (int)n : 1;
}

typedef void (*col_fn)(void *ctx, int64_t j0, int64_t j1);
typedef struct {
  col_fn fn;
  void *ctx;
  int64_t j0, j1;
} col_task;

static void *col_task_run(void *p) {
  col_task *t = (col_task *)p;
  if (t->j1 > t->j0) t->fn(t->ctx, t->j0, t->j1);
  return NULL;
}

/* Runs fn over columns [0, n) split into contiguous ranges, one per thread. */
static void parallel_cols(int64_t n, int nthreads, col_fn fn, void *ctx) {
  if (nthreads <= 0) nthreads = or_default_threads();
  if (nthreads > n) nthreads = (int)(n > 0 ? n : 1);
  if (nthreads <= 1) {
    if (n > 0) fn(ctx, 0, n);
    return;
  }
  pthread_t *th = (pthread_t *)malloc(sizeof(pthread_t) * nthreads);
  col_task *tk = (col_task *)malloc(sizeof(col_task) * nthreads);
  int64_t per = (n + nthreads - 1) / nthreads;
  for (int t = 0; t < nthreads; t++) {
    tk[t].fn = fn;
    tk[t].ctx = ctx;
    tk[t].j0 = (int64_t)t * per < n ? (int64_t)t * per : n;
    tk[t].j1 = (int64_t)(t + 1) * per < n ? (int64_t)(t + 1) * per : n;
    pthread_create(&th[t], NULL, col_task_run, &tk[t]);
  }
  for (int t = 0; t < nthreads; t++) pthread_join(th[t], NULL);
  free(th);
  free(tk);
}

/* ------------------------------------------------------------------------- */
/* seeded inputs — src/random/random.mjs:4-26                                 */
/* ------------------------------------------------------------------------- */

/* mulberry32 (random.mjs:4-12) in uint32 arithmetic: Math.imul and the int32
 * wrap of `(a + c) | 0` are both multiplication/addition mod 2^32, and every
 * `>>>` reads the same 32-bit pattern. */
double or_mulberry32_next(uint32_t *state) {
  uint32_t a = *state + 0x6d2b79f5u;
  *state = a;
  uint32_t t = (a ^ (a >> 15)) * (1u | a);
  t = (t + (t ^ (t >> 7)) * (61u | t)) ^ t;
  return (double)(t ^ (t >> 14)) / 4294967296.0;
}

/* random.mjs:14-19: the sum is formed in double, then stored into a Float32Array
 * (round to nearest even), which a C double->float conversion also does. */
void or_random_f32(float *out, int64_t n, double low, double high, uint32_t seed) {
  uint32_t s = seed;
  for (int64_t i = 0; i < n; i++) out[i] = (float)(low + or_mulberry32_next(&s) * (high - low));
}

void or_random_f64(double *out, int64_t n, double low, double high, uint32_t seed) {
  uint32_t s = seed;
  for (int64_t i = 0; i < n; i++) out[i] = low + or_mulberry32_next(&s) * (high - low);
}

/* Box-Muller on mulberry32 draws, two normals per pair of draws:
 *   r = sqrt(-2 ln(1 - u1)),  z0 = r cos(2 pi u2),  z1 = r sin(2 pi u2).
 * 1 - u1 lies in (0, 1], so the log is finite. */
static void normal_pairs(double *out, int64_t n, uint32_t seed) {
  uint32_t s = seed;
  const double two_pi = 6.283185307179586476925286766559;
  for (int64_t i = 0; i < n; i += 2) {
    double u1 = or_mulberry32_next(&s);
    double u2 = or_mulberry32_next(&s);
    double r = sqrt(-2.0 * log(1.0 - u1));
    out[i] = r * cos(two_pi * u2);
    if (i + 1 < n) out[i + 1] = r * sin(two_pi * u2);
  }
}

void or_random_normal_f64(double *out, int64_t n, uint32_t seed) { normal_pairs(out, n, seed); }

void or_random_normal_f32(float *out, int64_t n, uint32_t seed) {
  const int64_t chunk = 1 << 16;
  double *tmp = (double *)malloc(sizeof(double) * (size_t)(n < chunk ? (n > 0 ? n : 1) : chunk));
  /* Draw in chunks of an even size so the pair boundaries match one long stream. */
  uint32_t s = seed;
  const double two_pi = 6.283185307179586476925286766559;
  for (int64_t i0 = 0; i0 < n; i0 += chunk) {
    int64_t len = n - i0 < chunk ? n - i0 : chunk;
    for (int64_t i = 0; i < len; i += 2) {
      double u1 = or_mulberry32_next(&s);
      double u2 = or_mulberry32_next(&s);
      double r = sqrt(-2.0 * log(1.0 - u1));
      tmp[i] = r * cos(two_pi * u2);
      if (i + 1 < len) tmp[i + 1] = r * sin(two_pi * u2);
    }
    for (int64_t i = 0; i < len; i++) out[i0 + i] = (float)tmp[i];
  }
  free(tmp);
}

/* ------------------------------------------------------------------------- */
/* sgemm restatement — src/shaders/sgemm_large.wgsl:112-308                   */
/* ------------------------------------------------------------------------- */

typedef struct {
  int variant, transB;
  int64_t m, k;
  float alpha, beta;
  const float *Ap; /* op(A) packed column-major, m x k, ld = m */
  const float *B;
  int64_t ldb;
  float *C;
  int64_t ldc;
} sgemm_ctx;

#define OR_IB 64

/* Per element: acc = sum over p in increasing order (sgemm_large.wgsl:221-233,
 * the k tiles of :112 taken in order and each tile's dotIdx in order; zero-filled
 * tail entries add +0 and cannot change a non-(-0) sum), then the epilogue of
 * :299-304: acc2 = alpha==0 ? 0 : alpha*acc;  C = beta!=0 ? acc2 + beta*C : acc2. */
#define SGEMM_BODY(FMA_ACC, FMA_EPI)                                              \
  const sgemm_ctx *c = (const sgemm_ctx *)vctx;                                   \
  float acc[OR_IB];                                                               \
  for (int64_t j = j0; j < j1; j++) {                                             \
    for (int64_t i0 = 0; i0 < c->m; i0 += OR_IB) {                                \
      int64_t ib = c->m - i0 < OR_IB ? c->m - i0 : OR_IB;                         \
      for (int64_t ii = 0; ii < ib; ii++) acc[ii] = 0.0f;                         \
      if (c->alpha != 0.0f) {                                                     \
        for (int64_t p = 0; p < c->k; p++) {                                      \
          float b = c->transB ? c->B[j + p * c->ldb] : c->B[p + j * c->ldb];      \
          const float *a = c->Ap + i0 + p * c->m;                                 \
          for (int64_t ii = 0; ii < ib; ii++) acc[ii] = FMA_ACC(a[ii], b, acc[ii]);  \
        }                                                                         \
      }                                                                           \
      float *cc = c->C + i0 + j * c->ldc;                                         \
      for (int64_t ii = 0; ii < ib; ii++) {                                       \
        float s = (c->alpha == 0.0f) ? 0.0f : c->alpha * acc[ii];                 \
        cc[ii] = (c->beta != 0.0f) ? FMA_EPI(c->beta, cc[ii], s) : s;             \
      }                                                                           \
    }                                                                             \
  }

#define MUL_ADD(a, b, c) ((c) + (a) * (b))
#define FMA_F(a, b, c) fmaf((a), (b), (c))

static void sgemm_cols_unfused(void *vctx, int64_t j0, int64_t j1) { SGEMM_BODY(MUL_ADD, MUL_ADD) }

__attribute__((target("fma"))) static void sgemm_cols_fma_hw(void *vctx, int64_t j0, int64_t j1) {
  SGEMM_BODY(FMA_F, FMA_F)
}
static void sgemm_cols_fma_sw(void *vctx, int64_t j0, int64_t j1) { SGEMM_BODY(FMA_F, FMA_F) }

/* Copies op(A) (m x k) into a dense column-major buffer so the inner loop runs
 * along i for either transA; the values and the per-element order of the sum are
 * unchanged. */
static float *pack_opA_f32(int transA, int64_t m, int64_t k, const float *A, int64_t lda) {
  float *Ap = (float *)malloc(sizeof(float) * (size_t)(m * k > 0 ? m * k : 1));
  for (int64_t p = 0; p < k; p++)
    for (int64_t i = 0; i < m; i++) Ap[i + p * m] = transA ? A[p + i * lda] : A[i + p * lda];
  return Ap;
}

void or_sgemm(int variant, int transA, int transB, int64_t m, int64_t n, int64_t k,
              float alpha, const float *A, int64_t lda, const float *B, int64_t ldb,
              float beta, float *C, int64_t ldc, int nthreads) {
  if (m <= 0 || n <= 0) return; /* src/sgemm/sgemm.mjs:83 */
  float *Ap = (alpha != 0.0f && k > 0) ? pack_opA_f32(transA, m, k, A, lda) : NULL;
  sgemm_ctx ctx = {variant, transB, m, (alpha != 0.0f) ? k : 0, alpha, beta, Ap, B, ldb, C, ldc};
  col_fn fn = sgemm_cols_unfused;
  if (variant == 1) fn = __builtin_cpu_supports("fma") ? sgemm_cols_fma_hw : sgemm_cols_fma_sw;
  parallel_cols(n, nthreads, fn, &ctx);
  free(Ap);
}

typedef struct {
  int transA, transB;
  int64_t m, k;
  double alpha, beta;
  const void *A, *B, *C;
  int64_t lda, ldb, ldc;
  double *out, *absab;
  int64_t ldo;
} truth_ctx;

static void sgemm_truth_cols(void *vctx, int64_t j0, int64_t j1) {
  const truth_ctx *c = (const truth_ctx *)vctx;
  const float *A = (const float *)c->A, *B = (const float *)c->B, *C = (const float *)c->C;
  for (int64_t j = j0; j < j1; j++)
    for (int64_t i = 0; i < c->m; i++) {
      double acc = 0.0, ab = 0.0;
      for (int64_t p = 0; p < c->k; p++) {
        double a = c->transA ? A[p + i * c->lda] : A[i + p * c->lda];
        double b = c->transB ? B[j + p * c->ldb] : B[p + j * c->ldb];
        acc += a * b; /* exact product of two floats; one rounding per sum */
        ab += fabs(a) * fabs(b);
      }
      double s = (c->alpha == 0.0) ? 0.0 : c->alpha * acc;
      double r = (c->beta != 0.0) ? s + c->beta * (double)C[i + j * c->ldc] : s;
      c->out[i + j * c->ldo] = r;
      if (c->absab) c->absab[i + j * c->ldo] = ab;
    }
}

void or_sgemm_truth(int transA, int transB, int64_t m, int64_t n, int64_t k,
                    float alpha, const float *A, int64_t lda, const float *B, int64_t ldb,
                    float beta, const float *C, int64_t ldc,
                    double *out, double *absab, int64_t ldo, int nthreads) {
  if (m <= 0 || n <= 0) return;
  truth_ctx ctx = {transA, transB, m, k, alpha, beta, A, B, C, lda, ldb, ldc, out, absab, ldo};
  parallel_cols(n, nthreads, sgemm_truth_cols, &ctx);
}

/* ------------------------------------------------------------------------- */
/* double-double primitives — src/shaders/f64/utils/{add,multiply,batch}.wgsl */
/* ------------------------------------------------------------------------- */

/* isFiniteF (add.wgsl:24-26): exponent field not all ones. */
static int dd_finite(float x) {
  uint32_t u;
  memcpy(&u, &x, 4);
  return (u & 0x7f800000u) != 0x7f800000u;
}

/* twoSum (add.wgsl:88-98, the protected form; :30-35 unprotected): s = a+b, v = s-a, e = (a-(s-v)) + (b-v); e = 0 if s
 * is not finite. */
void or_dd_two_sum(float a, float b, float *hi, float *lo) {
  float s = a + b;
  float v = s - a;
  float e = (a - (s - v)) + (b - v);
  *hi = s;
  *lo = dd_finite(s) ? e : 0.0f;
}

/* fastTwoSum (add.wgsl:100-110): s = a+b, e = b-(s-a). */
void or_dd_fast_two_sum(float a, float b, float *hi, float *lo) {
  float s = a + b;
  float e = b - (s - a);
  *hi = s;
  *lo = dd_finite(s) ? e : 0.0f;
}

/* bitSplit (multiply.wgsl:17-30): hi keeps the sign, exponent and top 11
 * mantissa bits (mask 0xFFFFF000); lo = a - hi exactly. */
static void dd_bit_split(float a, float *hi, float *lo) {
  uint32_t u;
  memcpy(&u, &a, 4);
  u &= 0xFFFFF000u;
  float h;
  memcpy(&h, &u, 4);
  *hi = h;
  *lo = a - h;
}

/* twoProdBit (multiply.wgsl:32-45): s = a*b and its error by four partial
 * products of the bit-split halves; lo = -e, or 0 when s is not finite. */
void or_dd_two_prod_bit(float a, float b, float *hi, float *lo) {
  float s = a * b;
  float ah, al, bh, bl;
  dd_bit_split(a, &ah, &al);
  dd_bit_split(b, &bh, &bl);
  float e1 = s - ah * bh;
  float e2 = e1 - al * bh;
  float e3 = e2 - ah * bl;
  float e = e3 - al * bl;
  *hi = s;
  *lo = dd_finite(s) ? -e : 0.0f;
}

/* ddAdd (add.wgsl:112-116 / batch.wgsl:76-80). */
void or_dd_add(float ahi, float alo, float bhi, float blo, float *hi, float *lo) {
  float sh, sl;
  or_dd_two_sum(ahi, bhi, &sh, &sl);
  float lo_sum = alo + blo;
  or_dd_fast_two_sum(sh, sl + lo_sum, hi, lo);
}

/* ddMul (batch.wgsl:103-109, the op dgemm_small.wgsl:225 calls):
 * p = twoProdBit(a.hi, b.hi); x = finite(p.hi) ? p.lo + (a.hi*b.lo + a.lo*b.hi) : 0;
 * result = fastTwoSum(p.hi, x). */
static void dd_mul_v(int variant, float ahi, float alo, float bhi, float blo, float *hi, float *lo) {
  float ph, pl;
  or_dd_two_prod_bit(ahi, bhi, &ph, &pl);
  /* The cross terms are the one unprotected product-sum in ddMul; variant 1
   * contracts it into a fused multiply-add, as a contracting shader compiler may. */
  float cross_terms = variant ? fmaf(ahi, blo, alo * bhi) : ahi * blo + alo * bhi;
  float cross = dd_finite(ph) ? pl + cross_terms : 0.0f;
  or_dd_fast_two_sum(ph, cross, hi, lo);
}

void or_dd_mul(float ahi, float alo, float bhi, float blo, float *hi, float *lo) {
  dd_mul_v(0, ahi, alo, bhi, blo, hi, lo);
}

/* splitDoubleDouble (src/util/f64.mjs:15-17,33-43). */
static void dd_split1(double x, float *hi, float *lo) {
  float h = (float)x;
  *hi = h;
  *lo = isfinite(h) ? (float)(x - (double)h) : 0.0f;
}

void or_dd_split(const double *x, float *hi, float *lo, int64_t n) {
  for (int64_t i = 0; i < n; i++) dd_split1(x[i], &hi[i], &lo[i]);
}

void or_dd_merge(const float *hi, const float *lo, double *out, int64_t n) {
  for (int64_t i = 0; i < n; i++) out[i] = (double)hi[i] + (double)lo[i];
}

/* Object.is on floats: same bits, except that every NaN equals every NaN. */
static int same_f32(float a, float b) {
  if (isnan(a) && isnan(b)) return 1;
  uint32_t ua, ub;
  memcpy(&ua, &a, 4);
  memcpy(&ub, &b, 4);
  return ua == ub;
}

/* representable (f64.mjs:19-22). */
static int dd_representable(double v, float h, float l) {
  if (isfinite(v)) return fabs((double)h + (double)l - v) <= fabs(v) * 0x1p-40;
  if (isnan(v)) return isnan(h);
  return (double)h == v;
}

/* mergeDoubleDoubleExact (f64.mjs:80-91). */
static double dd_merge_exact1(float hi, float lo, double before) {
  float h, l;
  dd_split1(before, &h, &l);
  if (same_f32(hi, h) && same_f32(lo, l) && dd_representable(before, h, l)) return before;
  return (double)hi + (double)lo;
}

void or_dd_merge_exact(const float *hi, const float *lo, const double *before, double *out,
                       int64_t n) {
  for (int64_t i = 0; i < n; i++) out[i] = dd_merge_exact1(hi[i], lo[i], before[i]);
}

/* ------------------------------------------------------------------------- */
/* dgemm restatements                                                          */
/* ------------------------------------------------------------------------- */

typedef struct {
  int variant, transA, transB;
  int64_t m, k;
  float ahi, alo, bhi, blo; /* alpha, beta split (dgemm.mjs:233-238) */
  const float *Ahi, *Alo, *Bhi, *Blo; /* operands split like the host (dgemm.mjs:199-222) */
  int64_t lda, ldb;
  double *C;
  int64_t ldc;
} dd_ctx;

/* dgemm_small.wgsl:217-271 for one element, then the exact merge. */
static void dgemm_dd_cols(void *vctx, int64_t j0, int64_t j1) {
  const dd_ctx *c = (const dd_ctx *)vctx;
  const int alpha_zero = c->ahi == 0.0f && c->alo == 0.0f;
  const int beta_zero = c->bhi == 0.0f && c->blo == 0.0f;
  for (int64_t j = j0; j < j1; j++)
    for (int64_t i = 0; i < c->m; i++) {
      float acc_h = 0.0f, acc_l = 0.0f;
      for (int64_t p = 0; p < c->k; p++) {
        int64_t ia = c->transA ? p + i * c->lda : i + p * c->lda;
        int64_t ib = c->transB ? j + p * c->ldb : p + j * c->ldb;
        float mh, ml;
        dd_mul_v(c->variant, c->Ahi[ia], c->Alo[ia], c->Bhi[ib], c->Blo[ib], &mh, &ml);
        or_dd_add(acc_h, acc_l, mh, ml, &acc_h, &acc_l);
      }
      double *cp = c->C + i + j * c->ldc;
      const double before = *cp;
      float ch, cl;
      dd_split1(before, &ch, &cl);
      float sh, sl;
      dd_mul_v(c->variant, c->ahi, c->alo, acc_h, acc_l, &sh, &sl);
      if (alpha_zero) sh = sl = 0.0f;
      float th, tl;
      dd_mul_v(c->variant, c->bhi, c->blo, ch, cl, &th, &tl);
      float wh, wl;
      or_dd_add(sh, sl, th, tl, &wh, &wl);
      float oh = beta_zero ? sh : wh;
      float ol = beta_zero ? sl : wl;
      *cp = dd_merge_exact1(oh, ol, before);
    }
}

static void split_alloc(const double *x, int64_t n, float **hi, float **lo) {
  size_t sz = (size_t)(n > 0 ? n : 1);
  *hi = (float *)malloc(sizeof(float) * sz);
  *lo = (float *)malloc(sizeof(float) * sz);
  or_dd_split(x, *hi, *lo, n);
}

void or_dgemm_dd(int variant, int transA, int transB, int64_t m, int64_t n, int64_t k,
                 double alpha, const double *A, int64_t lda, const double *B, int64_t ldb,
                 double beta, double *C, int64_t ldc, int nthreads) {
  if (m <= 0 || n <= 0) return;                          /* dgemm.mjs:83 */
  if ((alpha == 0.0 || k == 0) && beta == 1.0) return;   /* dgemm.mjs:179 */
  int64_t nA = k > 0 ? (transA ? (m - 1) * lda + k : (k - 1) * lda + m) : 0;
  int64_t nB = k > 0 ? (transB ? (k - 1) * ldb + n : (n - 1) * ldb + k) : 0;
  float *Ahi, *Alo, *Bhi, *Blo;
  split_alloc(A, nA, &Ahi, &Alo);
  split_alloc(B, nB, &Bhi, &Blo);
  dd_ctx ctx;
  ctx.variant = variant;
  ctx.transA = transA;
  ctx.transB = transB;
  ctx.m = m;
  ctx.k = k;
  dd_split1(alpha, &ctx.ahi, &ctx.alo);
  dd_split1(beta, &ctx.bhi, &ctx.blo);
  ctx.Ahi = Ahi;
  ctx.Alo = Alo;
  ctx.Bhi = Bhi;
  ctx.Blo = Blo;
  ctx.lda = lda;
  ctx.ldb = ldb;
  ctx.C = C;
  ctx.ldc = ldc;
  parallel_cols(n, nthreads, dgemm_dd_cols, &ctx);
  free(Ahi);
  free(Alo);
  free(Bhi);
  free(Blo);
}

typedef struct {
  int transA, transB;
  int64_t m, k;
  double alpha, beta;
  const double *A, *B;
  int64_t lda, ldb;
  double *C;
  int64_t ldc;
} dfma_ctx;

static void dgemm_fma_cols(void *vctx, int64_t j0, int64_t j1) {
  const dfma_ctx *c = (const dfma_ctx *)vctx;
  for (int64_t j = j0; j < j1; j++)
    for (int64_t i = 0; i < c->m; i++) {
      double acc = 0.0;
      if (c->alpha != 0.0)
        for (int64_t p = 0; p < c->k; p++) {
          double a = c->transA ? c->A[p + i * c->lda] : c->A[i + p * c->lda];
          double b = c->transB ? c->B[j + p * c->ldb] : c->B[p + j * c->ldb];
          acc = fma(a, b, acc);
        }
      double *cp = c->C + i + j * c->ldc;
      double s = (c->alpha == 0.0) ? 0.0 : c->alpha * acc;
      *cp = (c->beta != 0.0) ? fma(c->beta, *cp, s) : s;
    }
}

void or_dgemm_fma(int transA, int transB, int64_t m, int64_t n, int64_t k,
                  double alpha, const double *A, int64_t lda, const double *B, int64_t ldb,
                  double beta, double *C, int64_t ldc, int nthreads) {
  if (m <= 0 || n <= 0) return;
  if ((alpha == 0.0 || k == 0) && beta == 1.0) return;
  dfma_ctx ctx = {transA, transB, m, k, alpha, beta, A, B, lda, ldb, C, ldc};
  parallel_cols(n, nthreads, dgemm_fma_cols, &ctx);
}

static void dgemm_truth_cols(void *vctx, int64_t j0, int64_t j1) {
  const truth_ctx *c = (const truth_ctx *)vctx;
  const double *A = (const double *)c->A, *B = (const double *)c->B, *C = (const double *)c->C;
  for (int64_t j = j0; j < j1; j++)
    for (int64_t i = 0; i < c->m; i++) {
      long double acc = 0.0L;
      double ab = 0.0;
      for (int64_t p = 0; p < c->k; p++) {
        double a = c->transA ? A[p + i * c->lda] : A[i + p * c->lda];
        double b = c->transB ? B[j + p * c->ldb] : B[p + j * c->ldb];
        acc += (long double)a * (long double)b;
        ab += fabs(a) * fabs(b);
      }
      long double s = (c->alpha == 0.0) ? 0.0L : (long double)c->alpha * acc;
      long double r = (c->beta != 0.0) ? s + (long double)c->beta * (long double)C[i + j * c->ldc] : s;
      c->out[i + j * c->ldo] = (double)r;
      if (c->absab) c->absab[i + j * c->ldo] = ab;
    }
}

void or_dgemm_truth(int transA, int transB, int64_t m, int64_t n, int64_t k,
                    double alpha, const double *A, int64_t lda, const double *B, int64_t ldb,
                    double beta, const double *C, int64_t ldc,
                    double *out, double *absab, int64_t ldo, int nthreads) {
  if (m <= 0 || n <= 0) return;
  truth_ctx ctx = {transA, transB, m, k, alpha, beta, A, B, C, lda, ldb, ldc, out, absab, ldo};
  parallel_cols(n, nthreads, dgemm_truth_cols, &ctx);
}
