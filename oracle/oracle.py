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
