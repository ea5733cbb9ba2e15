"""``sgemm`` / ``dgemm``: C := alpha*op(A)*op(B) + beta*C with wgblas's arguments.

Mirrors src/sgemm/sgemm.mjs:25-269 and src/dgemm/dgemm.mjs:23-318: the same
argument order, the same validation (in the same order, with the same
messages) and the same return shape —

* plain arrays (``Float32Array`` / ``Float64Array``, i.e. 1-D numpy arrays):
  returns ``{"C": new_array}`` (plus ``"gpuTimeMs"`` on a benchmark device);
  the input C is left unmodified;
* all-``GpuMatrix`` operands: C is updated in place and ``{}`` (or
  ``{"gpuTimeMs": t}``) is returned.

The call then maps the operands' layouts onto the column-major frame of the C
ABI (include/wgblas.h) — the counterpart of the row-major frame swap at
src/sgemm/sgemm.mjs:151-167 — and runs ``wg_sgemm`` / ``wg_dgemm`` (device
buffers) or ``wg_sgemm_host`` / ``wg_dgemm_host`` (host arrays). Calls are
synchronous: they return when C holds the result, as the reference's promise
resolves after readback.

The keyword ``out=`` (an extension) names the array to receive the result on
the plain-array path instead of a new one; pass a page-locked array from
``pinned_empty`` to read the result back at full PCIe rate.
"""
from __future__ import annotations

import ctypes as ct
import math

import numpy as np

from . import _native as nat
from ._runtime import Error, require_gpu_device, require_same_device
from .classes import GpuMatrix, _is_int, is_f32_array, is_f64_array

_TRANS = ("no-transpose", "transpose")
_UPLO = ("lower", "upper")
_LAYOUTS = ("row-major", "column-major")


def _is_number(x) -> bool:
    return isinstance(x, (int, float, np.integer, np.floating)) and not isinstance(x, (bool, np.bool_))


def _validate(routine, device, transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, layout, uplo=None):
    """The checks of src/sgemm/sgemm.mjs:42-149 (dgemm.mjs:40-149), in order; with
    ``uplo`` those of src/sgemmtr/sgemmtr.mjs:42-160 (the uplo check first).

    Returns None to proceed or the quick-return value for m == 0 or n == 0.
    """
    f64 = routine.startswith("d")
    is_arr = is_f64_array if f64 else is_f32_array
    arr_name = "Float64Array" if f64 else "Float32Array"
    a_gpu = isinstance(A, GpuMatrix)
    b_gpu = isinstance(B, GpuMatrix)
    c_gpu = isinstance(C, GpuMatrix)

    require_gpu_device(device)
    require_same_device(device, routine, {"A": A, "B": B, "C": C})
    if routine.endswith("gemmtr") and uplo not in _UPLO:
        raise Error("uplo must be 'lower' or 'upper'.")
    if transA not in _TRANS:
        raise Error("transA must be 'no-transpose' or 'transpose'.")
    if transB not in _TRANS:
        raise Error("transB must be 'no-transpose' or 'transpose'.")
    if layout not in _LAYOUTS:
        raise Error("layout must be 'row-major' or 'column-major'.")
    for name, v in (("alpha", alpha), ("beta", beta)):
        if not _is_number(v):
            raise Error(f"{name} must be a number.")
        if math.isnan(v):
            raise Error(f"{name} must not be NaN.")
        if not math.isfinite(v):
            raise Error(f"{name} must be finite.")
    if not all(_is_int(v) for v in (m, n, k, lda, ldb, ldc)):
        raise Error("m, n, k, lda, ldb, and ldc must be integers.")
    if not a_gpu and not is_arr(A):
        raise Error(f"A must be a {arr_name} or GpuMatrix.")
    if not b_gpu and not is_arr(B):
        raise Error(f"B must be a {arr_name} or GpuMatrix.")
    if not c_gpu and not is_arr(C):
        raise Error(f"C must be a {arr_name} or GpuMatrix.")
    if f64:
        for name, X, is_gpu in (("A", A, a_gpu), ("B", B, b_gpu), ("C", C, c_gpu)):
            if is_gpu and X.dtype is not np.float64:
                raise Error(f"{name} must be a Float64Array-backed GpuMatrix.")
    if (a_gpu or b_gpu) and not c_gpu:
        raise Error("C must be a GpuMatrix when A or B is a GpuMatrix.")
    if c_gpu and (not a_gpu or not b_gpu):
        raise Error("A and B must be GpuMatrix when C is a GpuMatrix.")
    if m < 0 or n < 0 or k < 0:
        raise Error("m, n, and k must be non-negative.")
    if lda <= 0 or ldb <= 0 or ldc <= 0:
        raise Error("lda, ldb, and ldc must be positive.")
    if m == 0 or n == 0:
        return {} if c_gpu else {"C": C}

    la = A.layout if a_gpu else layout
    lb = B.layout if b_gpu else layout
    lc = C.layout if c_gpu else layout

    # A: op(A) is m x k; the stored matrix is m x k or k x m by transA.
    a_rows, a_cols = (k, m) if la == "column-major" else (m, k)
    a_outer = a_rows if transA == "no-transpose" else a_cols
    a_inner = a_cols if transA == "no-transpose" else a_rows
    if lda < a_inner:
        raise Error(f"lda must be >= {'rows' if la == 'column-major' else 'cols'} of A as stored.")
    if a_gpu:
        if lda != A.lda:
            raise Error("lda must match A.lda when A is a GpuMatrix.")
        lr, lcl = (m, k) if transA == "no-transpose" else (k, m)
        if A.rows < lr or A.cols < lcl:
            raise Error("A is too small for the given m, k, and transA.")
    elif A.size < (a_outer - 1) * lda + a_inner:
        raise Error("A does not have enough elements for the given dimensions and lda.")

    # B: op(B) is k x n.
    b_rows, b_cols = (n, k) if lb == "column-major" else (k, n)
    b_outer = b_rows if transB == "no-transpose" else b_cols
    b_inner = b_cols if transB == "no-transpose" else b_rows
    if ldb < b_inner:
        raise Error(f"ldb must be >= {'rows' if lb == 'column-major' else 'cols'} of B as stored.")
    if b_gpu:
        if ldb != B.lda:
            raise Error("ldb must match B.lda when B is a GpuMatrix.")
        lr, lcl = (k, n) if transB == "no-transpose" else (n, k)
        if B.rows < lr or B.cols < lcl:
            raise Error("B is too small for the given n, k, and transB.")
    elif B.size < (b_outer - 1) * ldb + b_inner:
        raise Error("B does not have enough elements for the given dimensions and ldb.")

    # C: always m x n; layout decides the stored orientation.
    c_outer = n if lc == "column-major" else m
    c_inner = m if lc == "column-major" else n
    if ldc < c_inner:
        raise Error(f"ldc must be >= {'rows' if lc == 'column-major' else 'cols'} of C as stored.")
    if c_gpu:
        if ldc != C.lda:
            raise Error("ldc must match C.lda when C is a GpuMatrix.")
        if C.rows < m or C.cols < n:
            raise Error("C is too small for the given m and n.")
    elif C.size < (c_outer - 1) * ldc + c_inner:
        raise Error("C does not have enough elements for the given dimensions and ldc.")
    return None


def to_column_major_frame(transA, transB, m, n, A, lda, B, ldb, la, lb, lc):
    """Maps a call onto the column-major frame of the C ABI.

    A row-major stored matrix is the transpose of the column-major matrix with
    the same memory and leading dimension, so a row-major operand flips its
    trans flag; a row-major C is computed as C^T = op(B)^T op(A)^T, which swaps
    the operands and m/n and flips both flags (the column-major twin of
    src/sgemm/sgemm.mjs:151-167). Returns (tA, tB, m, n, A, lda, B, ldb).
    """
    ta = (transA == "transpose") == (la == "column-major")
    tb = (transB == "transpose") == (lb == "column-major")
    if lc == "column-major":
        return int(ta), int(tb), m, n, A, lda, B, ldb
    return int(not tb), int(not ta), n, m, B, ldb, A, lda


def _gemm(routine, device, transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, layout,
          out=None, uplo=None):
    early = _validate(routine, device, transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc,
                      layout, uplo)
    if early is not None:
        return early
    return _execute(routine.startswith("d"), device, transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C,
                    ldc, layout, out, uplo)


def _execute(f64, device, transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, layout, out=None,
             uplo=None):
    """Runs a validated call: the quick return, the layout mapping onto the
    column-major frame, and the C-ABI call (with ``uplo``, the gemmtr entry points)."""
    m, n, k, lda, ldb, ldc = (int(v) for v in (m, n, k, lda, ldb, ldc))
    if f64:
        alpha, beta = float(alpha), float(beta)
        # Reference BLAS quick return (src/dgemm/dgemm.mjs:177-179): C comes back as it is.
        if (alpha == 0 or k == 0) and beta == 1:
            return {} if isinstance(C, GpuMatrix) else {"C": C}
    else:
        # The reference passes alpha and beta to the kernel as f32 (src/sgemm/sgemm.mjs:191-192).
        alpha, beta = np.float32(alpha), np.float32(beta)
    c_gpu = isinstance(C, GpuMatrix)
    la = A.layout if c_gpu else layout
    lb = B.layout if c_gpu else layout
    lc = C.layout if c_gpu else layout
    ta, tb, mm, nn, AA, lda2, BB, ldb2 = to_column_major_frame(transA, transB, m, n, A, lda, B, ldb,
                                                               la, lb, lc)
    # The triangle is named in C's own (row, col) terms; a row-major C is computed
    # as C^T in the column-major frame, where it is the other triangle (the twin of
    # the column-major flip at src/sgemmtr/sgemmtr.mjs:178).
    tri = ()
    if uplo is not None:
        lower = (uplo == "lower") == (lc == "column-major")
        tri = (nat.WG_UPLO_LOWER if lower else nat.WG_UPLO_UPPER,)
    ms = ct.c_float(0.0)
    ms_p = ct.byref(ms) if device.benchmark else None
    if c_gpu:
        if uplo is None:
            fn = nat.lib.wg_dgemm if f64 else nat.lib.wg_sgemm
        else:
            fn = nat.lib.wg_dgemmtr if f64 else nat.lib.wg_sgemmtr
        nat.check(fn(device.handle, *tri, ta, tb, mm, nn, k, alpha, AA._buf, 0, lda2, BB._buf, 0, ldb2,
                     beta, C._buf, 0, ldc, ms_p))
        if not device.benchmark:
            nat.check(nat.lib.wg_device_sync(device.handle))
        device.check()
        return {"gpuTimeMs": float(ms.value)} if device.benchmark else {}
    # Plain arrays: the result is a new array (or `out`) — the input C is unchanged.
    if out is None:
        covered = (ldc == (m if lc == "column-major" else n)) and C.size == m * n
        out = np.empty_like(C) if covered else C.copy()
    elif not (isinstance(out, np.ndarray) and out.dtype == C.dtype and out.ndim == 1 and
              out.size >= C.size):
        raise Error("out must be a 1-D array of C's type and at least C's length.")
    if uplo is None:
        fn = nat.lib.wg_dgemm_host if f64 else nat.lib.wg_sgemm_host
    else:
        fn = nat.lib.wg_dgemmtr_host if f64 else nat.lib.wg_sgemmtr_host
    ptr = ct.c_void_p
    nat.check(fn(device.handle, *tri, ta, tb, mm, nn, k, alpha, ptr(AA.ctypes.data), lda2, ptr(BB.ctypes.data),
                 ldb2, beta, ptr(C.ctypes.data), ptr(out.ctypes.data), ldc, ms_p))
    device.check()
    res = {"C": out}
    if device.benchmark:
        res["gpuTimeMs"] = float(ms.value)
    return res


def sgemm(device, transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc,
          layout="row-major", *, out=None):
    """C := alpha*op(A)*op(B) + beta*C in fp32 (src/sgemm/sgemm.mjs:25-41)."""
    return _gemm("sgemm", device, transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, layout, out)


def dgemm(device, transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc,
          layout="row-major", *, out=None):
    """C := alpha*op(A)*op(B) + beta*C in native fp64 (src/dgemm/dgemm.mjs:23-39)."""
    return _gemm("dgemm", device, transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, layout, out)
