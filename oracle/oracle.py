"""ctypes front end of the CPU oracle (oracle.c) — TEST INFRASTRUCTURE ONLY.

Imported by tests/, by ``__graft_entry__.smoke()`` (as the checker) and by the
CPU-baseline legs of ``bench.py``. The product package never imports it.

All GEMM routines take numpy arrays in the column-major BLAS frame and the
reference's own argument meaning (trans flags as 0/1, leading dimensions in
elements). See oracle.h for the citations of the reference code each one
restates.
"""
from __future__ import annotations

import ctypes as ct
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

_i64 = ct.c_int64
_f32p = ct.POINTER(ct.c_float)
_f64p = ct.POINTER(ct.c_double)


def build(force: bool = False) -> str:
    """Compiles liboracle.so with oracle/Makefile (gcc)."""
    if force or not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < max(
        os.path.getmtime(os.path.join(_HERE, f)) for f in ("oracle.c", "oracle.h", "Makefile")
    ):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ct.CDLL(_LIB_PATH)
        L.or_mulberry32_next.argtypes = [ct.POINTER(ct.c_uint32)]
        L.or_mulberry32_next.restype = ct.c_double
        L.or_random_f32.argtypes = [_f32p, _i64, ct.c_double, ct.c_double, ct.c_uint32]
        L.or_random_f64.argtypes = [_f64p, _i64, ct.c_double, ct.c_double, ct.c_uint32]
        L.or_random_normal_f32.argtypes = [_f32p, _i64, ct.c_uint32]
        L.or_random_normal_f64.argtypes = [_f64p, _i64, ct.c_uint32]
        gemm_common = [ct.c_int, ct.c_int, _i64, _i64, _i64]
        L.or_sgemm.argtypes = [ct.c_int] + gemm_common + [
            ct.c_float, _f32p, _i64, _f32p, _i64, ct.c_float, _f32p, _i64, ct.c_int]
        L.or_sgemm_truth.argtypes = gemm_common + [
            ct.c_float, _f32p, _i64, _f32p, _i64, ct.c_float, _f32p, _i64,
            _f64p, _f64p, _i64, ct.c_int]
        L.or_dgemm_dd.argtypes = [ct.c_int] + gemm_common + [
            ct.c_double, _f64p, _i64, _f64p, _i64, ct.c_double, _f64p, _i64, ct.c_int]
        L.or_dgemm_fma.argtypes = gemm_common + [
            ct.c_double, _f64p, _i64, _f64p, _i64, ct.c_double, _f64p, _i64, ct.c_int]
        L.or_dgemm_truth.argtypes = gemm_common + [
            ct.c_double, _f64p, _i64, _f64p, _i64, ct.c_double, _f64p, _i64,
            _f64p, _f64p, _i64, ct.c_int]
        fpp = ct.POINTER(ct.c_float)
        for name in ("or_dd_two_sum", "or_dd_fast_two_sum", "or_dd_two_prod_bit"):
            getattr(L, name).argtypes = [ct.c_float, ct.c_float, fpp, fpp]
        for name in ("or_dd_add", "or_dd_mul"):
            getattr(L, name).argtypes = [ct.c_float] * 4 + [fpp, fpp]
        L.or_dd_split.argtypes = [_f64p, _f32p, _f32p, _i64]
        L.or_dd_merge.argtypes = [_f32p, _f32p, _f64p, _i64]
        L.or_dd_merge_exact.argtypes = [_f32p, _f32p, _f64p, _f64p, _i64]
        L.or_default_threads.restype = ct.c_int
        _lib = L
    return _lib


def _p32(a):
    return a.ctypes.data_as(_f32p)


def _p64(a):
    return a.ctypes.data_as(_f64p)


def _need(a, dtype):
    if not (isinstance(a, np.ndarray) and a.dtype == dtype and a.flags.c_contiguous):
        raise TypeError(f"expected a contiguous {np.dtype(dtype).name} array")
    return a


# ---- seeded inputs ---------------------------------------------------------

def random_f32(n, low=-1.0, high=1.0, seed=0):
    out = np.empty(n, np.float32)
    lib().or_random_f32(_p32(out), n, low, high, seed & 0xFFFFFFFF)
    return out


def random_f64(n, low=-1.0, high=1.0, seed=0):
    out = np.empty(n, np.float64)
    lib().or_random_f64(_p64(out), n, low, high, seed & 0xFFFFFFFF)
    return out


def normal_f32(n, seed=0):
    out = np.empty(n, np.float32)
    lib().or_random_normal_f32(_p32(out), n, seed & 0xFFFFFFFF)
    return out


def normal_f64(n, seed=0):
    out = np.empty(n, np.float64)
    lib().or_random_normal_f64(_p64(out), n, seed & 0xFFFFFFFF)
    return out


# ---- GEMM ------------------------------------------------------------------

def sgemm(transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, variant=1, threads=0):
    """Returns a new array: C after the reference's fp32 arithmetic (variant 1 = FMA)."""
    out = _need(C, np.float32).copy()
    lib().or_sgemm(variant, int(transA), int(transB), m, n, k, alpha,
                   _p32(_need(A, np.float32)), lda, _p32(_need(B, np.float32)), ldb,
                   beta, _p32(out), ldc, threads)
    return out


def sgemm_truth(transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, threads=0):
    """(truth, absab): fp64 result and sum|a||b|, dense column-major m x n."""
    truth = np.zeros(max(m * n, 1), np.float64)
    absab = np.zeros(max(m * n, 1), np.float64)
    lib().or_sgemm_truth(int(transA), int(transB), m, n, k, alpha,
                         _p32(_need(A, np.float32)), lda, _p32(_need(B, np.float32)), ldb,
                         beta, _p32(_need(C, np.float32)), ldc,
                         _p64(truth), _p64(absab), max(m, 1), threads)
    return truth[: m * n], absab[: m * n]


def dgemm_dd(transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, variant=0, threads=0):
    """Returns a new array: C after the reference's double-double dgemm (variant 0:
    every op rounded as written; 1: ddMul's cross terms fused)."""
    out = _need(C, np.float64).copy()
    lib().or_dgemm_dd(variant, int(transA), int(transB), m, n, k, alpha,
                      _p64(_need(A, np.float64)), lda, _p64(_need(B, np.float64)), ldb,
                      beta, _p64(out), ldc, threads)
    return out


def dgemm_fma(transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, threads=0):
    out = _need(C, np.float64).copy()
    lib().or_dgemm_fma(int(transA), int(transB), m, n, k, alpha,
                       _p64(_need(A, np.float64)), lda, _p64(_need(B, np.float64)), ldb,
                       beta, _p64(out), ldc, threads)
    return out


def dgemm_truth(transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, threads=0):
    truth = np.zeros(max(m * n, 1), np.float64)
    absab = np.zeros(max(m * n, 1), np.float64)
    lib().or_dgemm_truth(int(transA), int(transB), m, n, k, alpha,
                         _p64(_need(A, np.float64)), lda, _p64(_need(B, np.float64)), ldb,
                         beta, _p64(_need(C, np.float64)), ldc,
                         _p64(truth), _p64(absab), max(m, 1), threads)
    return truth[: m * n], absab[: m * n]


# ---- double-double primitives ------------------------------------------------

def _pair(fn, *args):
    hi, lo = ct.c_float(), ct.c_float()
    fn(*[ct.c_float(a) for a in args], ct.byref(hi), ct.byref(lo))
    return np.float32(hi.value), np.float32(lo.value)


def dd_two_sum(a, b):
    return _pair(lib().or_dd_two_sum, a, b)


def dd_two_prod_bit(a, b):
    return _pair(lib().or_dd_two_prod_bit, a, b)


def dd_add(ahi, alo, bhi, blo):
    return _pair(lib().or_dd_add, ahi, alo, bhi, blo)


def dd_mul(ahi, alo, bhi, blo):
    return _pair(lib().or_dd_mul, ahi, alo, bhi, blo)


def dd_split(x):
    x = np.ascontiguousarray(x, np.float64)
    hi = np.empty(x.size, np.float32)
    lo = np.empty(x.size, np.float32)
    lib().or_dd_split(_p64(x), _p32(hi), _p32(lo), x.size)
    return hi, lo


def dd_merge(hi, lo):
    out = np.empty(hi.size, np.float64)
    lib().or_dd_merge(_p32(_need(hi, np.float32)), _p32(_need(lo, np.float32)), _p64(out), hi.size)
    return out


def dd_merge_exact(hi, lo, before):
    out = np.empty(hi.size, np.float64)
    lib().or_dd_merge_exact(_p32(_need(hi, np.float32)), _p32(_need(lo, np.float32)),
                            _p64(_need(before, np.float64)), _p64(out), hi.size)
    return out


def default_threads() -> int:
    return lib().or_default_threads()


# ---- tolerance checkers ---------------------------------------------------------

def block(C, m, n, ld):
    """The m x n block of a column-major array with leading dimension ld, shape (m, n)."""
    if m == 0 or n == 0:
        return np.zeros((m, n), C.dtype)
    idx = np.arange(m)[:, None] + np.arange(n)[None, :] * ld
    return C[idx]


def dense(x, m, n):
    """A dense column-major m x n vector (as the *_truth routines return) as (m, n)."""
    return np.asarray(x).reshape(m, n, order="F")


def tri_merge(uplo, full, C, m, n, ldc):
    """gemmtr's write mask (src/shaders/sgemm_large.wgsl:293-297) in the
    column-major frame: the elements of `full` in the uplo triangle of the m x n
    block (1 = lower, j <= i; 2 = upper, j >= i), C's own values elsewhere."""
    out = np.array(C, copy=True)
    for j in range(n):
        lo, hi = (j, m) if uplo == 1 else (0, min(j + 1, m))
        if lo < hi:
            out[j * ldc + lo: j * ldc + hi] = full[j * ldc + lo: j * ldc + hi]
    return out


def sgemmtr(uplo, transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, variant=1, threads=0):
    """The reference's sgemmtr: sgemm's per-element arithmetic, written only in the triangle."""
    full = sgemm(transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, variant, threads)
    return tri_merge(uplo, full, _need(C, np.float32), m, n, ldc)


def dgemmtr_fma(uplo, transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, threads=0):
    """dgemmtr in native fp64 (sequential FMA per element), written only in the triangle."""
    full = dgemm_fma(transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, threads)
    return tri_merge(uplo, full, _need(C, np.float64), m, n, ldc)


def sgemm_bound(m, n, k, alpha, absab, beta, C, ldc):
    """Per-element north-star bound 2*K*2^-24*(|alpha||A||B| + |beta||C|), shape (m, n).

    K is taken as max(k, 1) so a k=0 call still allows the one rounding of beta*C.
    """
    cin = np.abs(block(C, m, n, ldc).astype(np.float64))
    return 2.0 * max(k, 1) * 2.0**-24 * (abs(alpha) * dense(absab, m, n) + abs(beta) * cin)


def dgemm_bound(m, n, k, alpha, absab, beta, C, ldc):
    """Per-element north-star bound 4*K*2^-53*(|alpha||A||B| + |beta||C|), shape (m, n)."""
    cin = np.abs(block(C, m, n, ldc))
    return 4.0 * max(k, 1) * 2.0**-53 * (abs(alpha) * dense(absab, m, n) + abs(beta) * cin)


def forward_factor(got, truth, m, n, k, alpha, absab, beta, C, ldc, eps, kplus, cmul):
    """The reference's own forwardFactor (tests/sgemm/helpers.js:23-56 with eps=2^-23,
    kplus=1, cmul=1; tests/dgemm/helpers.js:30-63 with eps=2^-48, kplus=2, cmul=3):
    max |got-truth| / (eps*((k+kplus)|alpha|sum|a||b| + cmul|beta||C|)); where that
    bound is 0 the element must match exactly, else the factor is infinite."""
    g = block(got, m, n, ldc).astype(np.float64)
    cin = np.abs(block(C, m, n, ldc).astype(np.float64))
    err = np.abs(g - dense(truth, m, n))
    bound = eps * ((k + kplus) * abs(alpha) * dense(absab, m, n) + cmul * abs(beta) * cin)
    zero = bound == 0
    if np.any(err[zero] != 0):
        return float("inf")
    if np.all(zero):
        return 0.0
    return float(np.max(err[~zero] / bound[~zero]))


# ---- strsm: the reference's own test oracle, restated -----------------------------

def _index_grid(rows, cols, ld, layout):
    """Flat indices of a rows x cols matrix stored with leading dimension ld, shape (rows, cols)."""
    i = np.arange(rows)[:, None]
    j = np.arange(cols)[None, :]
    return (j * ld + i) if layout == "column-major" else (i * ld + j)


def tri_dense(A, lda, order, uplo, transA, diag, layout="row-major"):
    """op(A) as a dense float64 (order, order) matrix: denseTriangular of
    tests/helpers/stdlib.js:607-641. The stored `uplo` triangle (read with op
    applied), zeros outside it, ones on the diagonal for diag 'unit' (A's
    diagonal then unread); elements outside the triangle are never read."""
    A = np.asarray(A)
    out = np.zeros((order, order))
    if order == 0:
        return out
    i, j = np.meshgrid(np.arange(order), np.arange(order), indexing="ij")
    nt = transA == "no-transpose"
    lower = uplo == "lower"
    meaningful = ((j <= i) if lower else (j >= i)) if nt else ((j >= i) if lower else (j <= i))
    r, c = (i, j) if nt else (j, i)
    idx = (c * lda + r) if layout == "column-major" else (r * lda + c)
    off = meaningful & (i != j)
    out[off] = A[idx[off]].astype(np.float64)
    d = np.arange(order)
    if diag == "unit":
        out[d, d] = 1.0
    else:
        out[d, d] = A[idx[d, d]].astype(np.float64)
    return out


def strsm(side, uplo, transA, diag, m, n, alpha, A, lda, B, ldb, layout="row-major"):
    """strsmReference / solveTriangular of tests/helpers/stdlib.js:692-775: B's
    m x n block replaced by X with op(A)*X = alpha*B (side 'left') or
    X*op(A) = alpha*B ('right'), by row (left) or column (right) substitution.
    Each unknown is alpha*b minus the products with the unknowns already found,
    subtracted one at a time in f64 (the reference's JavaScript numbers), divided
    by the diagonal in f64 and stored rounded to f32; alpha = 0 gives zeros
    (the whole array, as the reference returns a fresh zero array). Returns a
    new float32 array the size of B; the padding keeps B's values."""
    B = np.asarray(B, np.float32)
    if alpha == 0:
        return np.zeros(B.size, np.float32)
    if m == 0 or n == 0:
        return B.copy()
    order = m if side == "left" else n
    D = tri_dense(A, lda, order, uplo, transA, diag, layout)
    op_lower = (transA == "no-transpose") == (uplo == "lower")
    idx = _index_grid(m, n, ldb, layout)
    Bm = B[idx].astype(np.float64)
    out = Bm.copy()
    with np.errstate(all="ignore"):
        for step in range(order):
            if side == "left":
                i = step if op_lower else order - 1 - step
                ks = np.arange(0, i) if op_lower else np.arange(i + 1, order)
                terms = np.empty((len(ks) + 1, n))
                terms[0] = alpha * Bm[i]
                terms[1:] = -(D[i, ks][:, None] * out[ks, :])
                acc = np.cumsum(terms, axis=0)[-1]  # strictly sequential, like the loop
                out[i] = (acc / D[i, i]).astype(np.float32)
            else:
                j = order - 1 - step if op_lower else step
                ks = np.arange(j + 1, order) if op_lower else np.arange(0, j)
                terms = np.empty((len(ks) + 1, m))
                terms[0] = alpha * Bm[:, j]
                terms[1:] = -(out[:, ks].T * D[ks, j][:, None])
                acc = np.cumsum(terms, axis=0)[-1]
                out[:, j] = (acc / D[j, j]).astype(np.float32)
    res = B.copy()
    res[idx] = out.astype(np.float32)
    return res


def strsm_residual_factor(X, side, uplo, transA, diag, m, n, alpha, A, lda, B, ldb, layout="row-major"):
    """backwardResidualFactor of tests/strsm/helpers.js: max over the m x n block of
    |op(A)*X - alpha*B| / (2^-23 * (order + 1) * |op(A)||X|) (X*op(A) for side
    'right'), with alpha*B taken as 0 when alpha = 0; where the bound is 0 the
    residual must be exactly 0, else the factor is infinite. The reference's
    strsm tests require a factor <= 5."""
    if m == 0 or n == 0:
        return 0.0
    order = m if side == "left" else n
    D = tri_dense(A, lda, order, uplo, transA, diag, layout)
    idx = _index_grid(m, n, ldb, layout)
    Xm = np.asarray(X)[idx].astype(np.float64)
    Bm = np.asarray(B)[idx].astype(np.float64)
    if side == "left":
        acc, dot = D @ Xm, np.abs(D) @ np.abs(Xm)
    else:
        acc, dot = Xm @ D, np.abs(Xm) @ np.abs(D)
    rhs = np.zeros_like(Bm) if alpha == 0 else alpha * Bm
    err = np.abs(acc - rhs)
    bound = 2.0**-23 * (order + 1) * dot
    zero = bound == 0
    if np.any(err[zero] != 0):
        return float("inf")
    if np.all(zero):
        return 0.0
    return float(np.max(err[~zero] / bound[~zero]))


# ---- sgemv / dgemv: the reference's test oracle, restated ---------------------------

def _mat_at(A, lda, layout):
    """A(i, j) of a matrix stored row- or column-major with leading dimension lda."""
    return (lambda i, j: A[j * lda + i]) if layout == "column-major" else (lambda i, j: A[i * lda + j])


def gemv(trans, m, n, alpha, A, lda, x, incx, beta, y, incy, layout="row-major"):
    """y := alpha*op(A)*x + beta*y as the reference's tests compute it: the
    published algorithm of @stdlib/blas-base-sgemv@0.1.1 / -dgemv@0.1.1 (npm
    dependencies not vendored in the reference, called at
    tests/helpers/stdlib.js:104-122,304-313), which is reference BLAS xGEMV:

    * m = 0, n = 0, or alpha = 0 with beta = 1: y unchanged;
    * y := beta*y first (zeros when beta = 0, y not read), then nothing more
      when alpha = 0;
    * the inner loop runs along A's storage: where op(A)'s rows are contiguous
      (row-major no-transpose, column-major transpose) each y entry gets
      temp = sum of A*x in increasing order, then y += alpha*temp; otherwise
      column by column, temp = alpha*x_j and y += temp*A(:, j), a column whose
      x entry is 0 skipped (tests/sgemv/src/test.sgemv.js:341-344).

    Every operation rounds to the array's type (f32 for float32 inputs, f64 for
    float64), as stdlib rounds each f32 step. Returns a new array the size of y;
    entries outside the strided y keep their values."""
    y = np.array(y, copy=True)
    dt = y.dtype.type
    if m == 0 or n == 0 or (alpha == 0 and beta == 1):
        return y
    A = np.asarray(A, dt)
    x = np.asarray(x, dt)
    no_t = trans == "no-transpose"
    xlen, ylen = (n, m) if no_t else (m, n)
    iy = np.arange(ylen) * incy
    ix = np.arange(xlen) * incx
    a, b = dt(alpha), dt(beta)
    with np.errstate(all="ignore"):
        if beta != 1:
            y[iy] = dt(0) if beta == 0 else b * y[iy]
        if alpha == 0:
            return y
        at = _mat_at(A, lda, layout)
        rows_contiguous = no_t == (layout != "column-major")
        yv = y[iy]
        if rows_contiguous:  # dot products: temp over the contraction index, in order
            temp = np.zeros(ylen, dt)
            for p in range(xlen):
                col = at(np.arange(ylen), p) if no_t else at(p, np.arange(ylen))
                temp = temp + col * x[ix[p]]
            yv = yv + a * temp
        else:  # column by column, skipping zero x entries
            for p in range(xlen):
                xp = x[ix[p]]
                if xp == 0:
                    continue
                t = a * xp
                col = at(np.arange(ylen), p) if no_t else at(p, np.arange(ylen))
                yv = yv + t * col
        y[iy] = yv
    return y


def gemv_forward_factor(got, ref, trans, m, n, alpha, A, lda, x, incx, beta, y, incy, layout="row-major"):
    """forwardFactor of tests/sgemv/helpers.js (eps = 2^-23) and tests/dgemv/helpers.js
    (eps = 2^-48), chosen by y's type: max over outputs of |got - ref| /
    (eps*((nTerms + 1)|alpha| sum|A||x| + |beta||y_in|)); an output whose bound is 0
    must match exactly, else the factor is infinite."""
    y = np.asarray(y)
    eps = 2.0**-48 if y.dtype == np.float64 else 2.0**-23
    no_t = trans == "no-transpose"
    xlen, ylen = (n, m) if no_t else (m, n)
    if ylen == 0 or xlen == 0:
        return 0.0
    at = _mat_at(np.abs(np.asarray(A, np.float64)), lda, layout)
    xa = np.abs(np.asarray(x, np.float64)[np.arange(xlen) * incx])
    i = np.arange(ylen)[:, None]
    p = np.arange(xlen)[None, :]
    mat = at(i, p) if no_t else at(p, i)
    dot = mat @ xa
    iy = np.arange(ylen) * incy
    err = np.abs(np.asarray(got, np.float64)[iy] - np.asarray(ref, np.float64)[iy])
    bound = eps * ((xlen + 1) * abs(alpha) * dot + abs(beta) * np.abs(y[iy].astype(np.float64)))
    zero = bound == 0
    if np.any(err[zero] != 0):
        return float("inf")
    if np.all(zero):
        return 0.0
    return float(np.max(err[~zero] / bound[~zero]))
