"""The gemmtr family: ``sgemmtr`` / ``dgemmtr``, ``ssyrk`` / ``dsyrk`` and
``ssyr2k`` / ``dsyr2k``, with wgblas's arguments.

Mirrors src/sgemmtr/sgemmtr.mjs, src/ssyrk/ssyrk.mjs and src/ssyr2k/ssyr2k.mjs
(and their d twins): the same argument order, validation order and messages,
and return shapes as ``sgemm`` / ``dgemm``. Only the ``uplo`` triangle of C
(``'lower'``: col <= row, ``'upper'``: col >= row, in C's own terms) is read or
written. As in the reference, the rank-k updates are compositions of gemmtr:

* ``ssyrk``: C := uplo(alpha*op(A)*op(A)^T + beta*C) is gemmtr with B := A and
  the opposite transpose (src/ssyrk/ssyrk.mjs:29-31);
* ``ssyr2k``: C := uplo(alpha*op(A)*op(B)^T + alpha*op(B)*op(A)^T + beta*C) is
  two gemmtr passes, the second with beta = 1 (src/ssyr2k/ssyr2k.mjs:25-26).

The d variants compute in native fp64 and keep the reference BLAS quick return
((alpha == 0 or k == 0) and beta == 1 leaves C as it is).
"""
from __future__ import annotations

import math

import numpy as np

from ._runtime import Error, require_gpu_device, require_same_device
from .classes import GpuMatrix, _is_int, is_f32_array, is_f64_array
from .gemm import _LAYOUTS, _TRANS, _UPLO, _execute, _gemm, _is_number


def sgemmtr(device, uplo, transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc,
            layout="row-major", *, out=None):
    """C := uplo(alpha*op(A)*op(B) + beta*C) in fp32 (src/sgemmtr/sgemmtr.mjs:25-41)."""
    return _gemm("sgemmtr", device, transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, layout, out,
                 uplo)


def dgemmtr(device, uplo, transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc,
            layout="row-major", *, out=None):
    """C := uplo(alpha*op(A)*op(B) + beta*C) in native fp64 (src/dgemmtr/dgemmtr.mjs)."""
    return _gemm("dgemmtr", device, transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, layout, out,
                 uplo)


def _validate_rank(routine, device, uplo, trans, n, k, alpha, A, lda, B, ldb, beta, C, ldc, layout):
    """The checks of src/ssyrk/ssyrk.mjs:42-123 (B is None) and
    src/ssyr2k/ssyr2k.mjs:47-141, in order. Returns None to proceed or the
    quick-return value for n == 0."""
    f64 = routine.startswith("d")
    is_arr = is_f64_array if f64 else is_f32_array
    arr_name = "Float64Array" if f64 else "Float32Array"
    two = B is not None or routine.endswith("2k")
    mats = {"A": A, "B": B, "C": C} if two else {"A": A, "C": C}
    a_gpu = isinstance(A, GpuMatrix)
    b_gpu = isinstance(B, GpuMatrix)
    c_gpu = isinstance(C, GpuMatrix)

    require_gpu_device(device)
    require_same_device(device, routine, mats)
    if uplo not in _UPLO:
        raise Error("uplo must be 'lower' or 'upper'.")
    if trans not in _TRANS:
        raise Error("trans must be 'no-transpose' or 'transpose'.")
    if layout not in _LAYOUTS:
        raise Error("layout must be 'row-major' or 'column-major'.")
    for name, v in (("alpha", alpha), ("beta", beta)):
        if not _is_number(v):
            raise Error(f"{name} must be a number.")
        if math.isnan(v):
            raise Error(f"{name} must not be NaN.")
        if not math.isfinite(v):
            raise Error(f"{name} must be finite.")
    if two:
        if not all(_is_int(v) for v in (n, k, lda, ldb, ldc)):
            raise Error("n, k, lda, ldb, and ldc must be integers.")
    elif not all(_is_int(v) for v in (n, k, lda, ldc)):
        raise Error("n, k, lda, and ldc must be integers.")
    if not a_gpu and not is_arr(A):
        raise Error(f"A must be a {arr_name} or GpuMatrix.")
    if two and not b_gpu and not is_arr(B):
        raise Error(f"B must be a {arr_name} or GpuMatrix.")
    if not c_gpu and not is_arr(C):
        raise Error(f"C must be a {arr_name} or GpuMatrix.")
    if f64:
        for name, X, is_gpu in (("A", A, a_gpu), ("B", B, b_gpu), ("C", C, c_gpu)):
            if is_gpu and X.dtype is not np.float64:
                raise Error(f"{name} must be a Float64Array-backed GpuMatrix.")
    if two:
        if (a_gpu or b_gpu) and not c_gpu:
            raise Error("C must be a GpuMatrix when A or B is a GpuMatrix.")
        if c_gpu and (not a_gpu or not b_gpu):
            raise Error("A and B must be GpuMatrix when C is a GpuMatrix.")
    else:
        if a_gpu and not c_gpu:
            raise Error("C must be a GpuMatrix when A is a GpuMatrix.")
        if c_gpu and not a_gpu:
            raise Error("A must be a GpuMatrix when C is a GpuMatrix.")
    if n < 0 or k < 0:
        raise Error("n and k must be non-negative.")
    if two:
        if lda <= 0 or ldb <= 0 or ldc <= 0:
            raise Error("lda, ldb, and ldc must be positive.")
    elif lda <= 0 or ldc <= 0:
        raise Error("lda and ldc must be positive.")
    if n == 0:
        return {} if c_gpu else {"C": C}

    # op(X) is n x k; the stored matrix is n x k or k x n by trans (both operands
    # share one trans, as netlib's syr2k does).
    for name, X, ldx, is_gpu in (("A", A, lda, a_gpu), ("B", B, ldb, b_gpu)) if two else (("A", A, lda, a_gpu),):
        lx = X.layout if is_gpu else layout
        rows, cols = (k, n) if lx == "column-major" else (n, k)
        outer = rows if trans == "no-transpose" else cols
        inner = cols if trans == "no-transpose" else rows
        if ldx < inner:
            raise Error(f"ld{name.lower()} must be >= {'rows' if lx == 'column-major' else 'cols'} of {name} as stored.")
        if is_gpu:
            if ldx != X.lda:
                raise Error(f"ld{name.lower()} must match {name}.lda when {name} is a GpuMatrix.")
            lr, lcl = (n, k) if trans == "no-transpose" else (k, n)
            if X.rows < lr or X.cols < lcl:
                raise Error(f"{name} is too small for the given n, k, and trans.")
        elif X.size < (outer - 1) * ldx + inner:
            raise Error(f"{name} does not have enough elements for the given dimensions and ld{name.lower()}.")
    # C: always n x n — layout only affects storage order, not size.
    if ldc < n:
        raise Error("ldc must be >= n.")
    if c_gpu:
        if ldc != C.lda:
            raise Error("ldc must match C.lda when C is a GpuMatrix.")
        if C.rows < n or C.cols < n:
            raise Error("C is too small for the given n.")
    elif C.size < (n - 1) * ldc + n:
        raise Error("C does not have enough elements for the given dimensions and ldc.")
    return None


def _flip(trans):
    return "no-transpose" if trans == "transpose" else "transpose"


def _rank_update(routine, device, uplo, trans, n, k, alpha, A, lda, B, ldb, beta, C, ldc, layout, out):
    early = _validate_rank(routine, device, uplo, trans, n, k, alpha, A, lda, B, ldb, beta, C, ldc, layout)
    if early is not None:
        return early
    f64 = routine.startswith("d")
    if f64 and (alpha == 0 or k == 0) and beta == 1:
        # Reference BLAS quick return (src/dsyrk/dsyrk.mjs:140-142, src/dsyr2k/dsyr2k.mjs:172-174).
        return {} if isinstance(C, GpuMatrix) else {"C": C}
    if B is None:
        # syrk: op(A) * op(A)^T is gemmtr with B := A and the other transpose.
        return _execute(f64, device, trans, _flip(trans), n, n, k, alpha, A, lda, A, lda, beta, C, ldc, layout,
                        out, uplo)
    # syr2k: two gemmtr passes, the second accumulating with beta = 1.
    first = _execute(f64, device, trans, _flip(trans), n, n, k, alpha, A, lda, B, ldb, beta, C, ldc, layout, None,
                     uplo)
    mid = C if isinstance(C, GpuMatrix) else first["C"]
    second = _execute(f64, device, trans, _flip(trans), n, n, k, alpha, B, ldb, A, lda, 1.0, mid, ldc, layout,
                      out, uplo)
    if "gpuTimeMs" in second:
        second["gpuTimeMs"] += first.get("gpuTimeMs", 0.0)
    return second


def ssyrk(device, uplo, trans, n, k, alpha, A, lda, beta, C, ldc, layout="row-major", *, out=None):
    """C := uplo(alpha*op(A)*op(A)^T + beta*C) in fp32 (src/ssyrk/ssyrk.mjs:29-43)."""
    return _rank_update("ssyrk", device, uplo, trans, n, k, alpha, A, lda, None, None, beta, C, ldc, layout, out)


def dsyrk(device, uplo, trans, n, k, alpha, A, lda, beta, C, ldc, layout="row-major", *, out=None):
    """C := uplo(alpha*op(A)*op(A)^T + beta*C) in native fp64 (src/dsyrk/dsyrk.mjs)."""
    return _rank_update("dsyrk", device, uplo, trans, n, k, alpha, A, lda, None, None, beta, C, ldc, layout, out)


def ssyr2k(device, uplo, trans, n, k, alpha, A, lda, B, ldb, beta, C, ldc, layout="row-major", *, out=None):
    """C := uplo(alpha*op(A)*op(B)^T + alpha*op(B)*op(A)^T + beta*C) in fp32
    (src/ssyr2k/ssyr2k.mjs:25-46)."""
    return _rank_update("ssyr2k", device, uplo, trans, n, k, alpha, A, lda, B, ldb, beta, C, ldc, layout, out)


def dsyr2k(device, uplo, trans, n, k, alpha, A, lda, B, ldb, beta, C, ldc, layout="row-major", *, out=None):
    """C := uplo(alpha*op(A)*op(B)^T + alpha*op(B)*op(A)^T + beta*C) in native fp64
    (src/dsyr2k/dsyr2k.mjs)."""
    return _rank_update("dsyr2k", device, uplo, trans, n, k, alpha, A, lda, B, ldb, beta, C, ldc, layout, out)
