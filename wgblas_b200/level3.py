"""``ssymm`` / ``dsymm``, ``strmm`` / ``dtrmm`` and ``strsm`` with wgblas's arguments.

Mirrors src/ssymm/ssymm.mjs, src/strmm/strmm.mjs (and the d twins) and
src/strsm/strsm.mjs: the same argument order, validation order and messages,
and return shapes. As in the reference, symm and trmm run as a pass that
materializes a dense copy of the special operand followed by a plain GEMM on
this library's kernels:

* symm: ``wg_symmetrize`` mirrors A's stored ``uplo`` triangle into a dense
  matrix, then C := alpha*A*B + beta*C (side 'left') or alpha*B*A + beta*C
  ('right');
* trmm: ``wg_triangularize`` builds op(A) densely (zeros outside the stored
  triangle, ones on the diagonal for ``diag='unit'``), the GEMM writes
  alpha*op(A)*B (or alpha*B*op(A)) into a scratch matrix with B's layout, and the
  block is copied back over B (B's leading-dimension padding is untouched).

strsm is one call of ``wg_strsm``: a recursive blocked triangular solve in place
on B, with substitution kernels on the 64-row diagonal blocks and GEMM updates
between them.

Plain arrays come back as new arrays (``{"C": ...}`` / ``{"B": ...}``); GpuMatrix
operands are updated in place. The d variants compute in native fp64; dsymm
keeps the BLAS quick return (alpha == 0 and beta == 1).
"""
from __future__ import annotations

import ctypes as ct
import math

import numpy as np

from . import _native as nat
from ._runtime import Error, require_gpu_device, require_same_device
from .classes import GpuMatrix, _is_int, is_f32_array, is_f64_array
from .gemm import _LAYOUTS, _TRANS, _UPLO, _execute, _is_number

_SIDES = ("left", "right")
_DIAGS = ("unit", "non-unit")


def _check_numbers(*pairs):
    for name, v in pairs:
        if not _is_number(v):
            raise Error(f"{name} must be a number.")
        if math.isnan(v):
            raise Error(f"{name} must not be NaN.")
        if not math.isfinite(v):
            raise Error(f"{name} must be finite.")


def _check_square(name, X, is_gpu, ld, order, side):
    """The symmetric / triangular operand's checks (src/ssymm/ssymm.mjs, order = m or n by side)."""
    if ld < order:
        raise Error(f"ld{name.lower()} must be >= " + ("m" if side == "left" else "n") + ".")
    if is_gpu:
        if ld != X.lda:
            raise Error(f"ld{name.lower()} must match {name}.lda when {name} is a GpuMatrix.")
        if X.rows < order or X.cols < order:
            raise Error(f"{name} is too small for the given m/n and side.")
    elif X.size < (order - 1) * ld + order:
        raise Error(f"{name} does not have enough elements for the given dimensions and ld{name.lower()}.")


def _check_general(name, X, is_gpu, ld, layout, m, n):
    """An m x n general operand (B or C): the rules of sgemm's C."""
    outer, inner = (n, m) if layout == "column-major" else (m, n)
    if ld < inner:
        raise Error(f"ld{name.lower()} must be >= {'rows' if layout == 'column-major' else 'cols'} of {name} as stored.")
    if is_gpu:
        if ld != X.lda:
            raise Error(f"ld{name.lower()} must match {name}.lda when {name} is a GpuMatrix.")
        if X.rows < m or X.cols < n:
            raise Error(f"{name} is too small for the given m and n.")
    elif X.size < (outer - 1) * ld + inner:
        raise Error(f"{name} does not have enough elements for the given dimensions and ld{name.lower()}.")


def _upload(device, arr, rows, cols, ld, layout):
    """A scratch GpuMatrix holding a plain array as stored (padding included; the
    last row or column may be short, as the reference's minimum sizes allow)."""
    outer = rows if layout == "row-major" else cols
    nbytes = outer * ld * arr.itemsize
    buf = nat.c_buf_p()
    nat.check(nat.lib.wg_buffer_alloc(device.handle, max(nbytes, 1), ct.byref(buf)))
    avail = min(arr.size, outer * ld) * arr.itemsize
    try:
        nat.check(nat.lib.wg_buffer_upload(buf, 0, arr.ctypes.data_as(ct.c_void_p), avail))
    except Exception:
        nat.lib.wg_buffer_free(buf)
        raise
    return GpuMatrix(buf, rows, cols, ld, None, layout, device, arr.dtype)


def _download_into(G, arr):
    """The bytes of a scratch GpuMatrix back over a copy of the plain array it came from."""
    out = arr.copy()
    outer = G.rows if G.layout == "row-major" else G.cols
    avail = min(out.size, outer * G.lda) * out.itemsize
    nat.check(nat.lib.wg_buffer_download(G._buf, 0, out.ctypes.data_as(ct.c_void_p), avail))
    return out


def _validate_special(routine, device, side, uplo, transA, diag, m, n, alpha, A, lda, B, ldb, beta, C, ldc, layout):
    """The checks of src/ssymm/ssymm.mjs:46-118 (C given) or src/strmm/strmm.mjs:51-113
    and src/strsm/strsm.mjs:174-240 (transA and diag given), in order. Returns None
    to proceed or the quick-return value."""
    trmm = C is None and routine.endswith(("trmm", "trsm"))
    f64 = routine.startswith("d")
    is_arr = is_f64_array if f64 else is_f32_array
    arr_name = "Float64Array" if f64 else "Float32Array"
    a_gpu, b_gpu, c_gpu = (isinstance(X, GpuMatrix) for X in (A, B, C))
    require_gpu_device(device)
    require_same_device(device, routine, {"A": A, "B": B} if trmm else {"A": A, "B": B, "C": C})
    if side not in _SIDES:
        raise Error("side must be 'left' or 'right'.")
    if uplo not in _UPLO:
        raise Error("uplo must be 'lower' or 'upper'.")
    if trmm:
        if transA not in _TRANS:
            raise Error("transA must be 'no-transpose' or 'transpose'.")
        if diag not in _DIAGS:
            raise Error("diag must be 'unit' or 'non-unit'.")
    if layout not in _LAYOUTS:
        raise Error("layout must be 'row-major' or 'column-major'.")
    _check_numbers(("alpha", alpha)) if trmm else _check_numbers(("alpha", alpha), ("beta", beta))
    ints = (m, n, lda, ldb) if trmm else (m, n, lda, ldb, ldc)
    if not all(_is_int(v) for v in ints):
        raise Error("m, n, lda, and ldb must be integers." if trmm else "m, n, lda, ldb, and ldc must be integers.")
    if not a_gpu and not is_arr(A):
        raise Error(f"A must be a {arr_name} or GpuMatrix.")
    if not b_gpu and not is_arr(B):
        raise Error(f"B must be a {arr_name} or GpuMatrix.")
    if not trmm and not c_gpu and not is_arr(C):
        raise Error(f"C must be a {arr_name} or GpuMatrix.")
    if f64:
        for name, X, is_gpu in (("A", A, a_gpu), ("B", B, b_gpu), ("C", C, c_gpu)):
            if is_gpu and X.dtype is not np.float64:
                raise Error(f"{name} must be a Float64Array-backed GpuMatrix.")
    if trmm:
        if a_gpu != b_gpu:
            raise Error("A and B must both be GpuMatrix or both be " + arr_name + ".")
    else:
        if (a_gpu or b_gpu) and not c_gpu:
            raise Error("C must be a GpuMatrix when A or B is a GpuMatrix.")
        if c_gpu and (not a_gpu or not b_gpu):
            raise Error("A and B must be GpuMatrix when C is a GpuMatrix.")
    if m < 0 or n < 0:
        raise Error("m and n must be non-negative.")
    if m == 0 or n == 0:
        if trmm:
            return {} if b_gpu else {"B": B}
        return {} if c_gpu else {"C": C}
    order = m if side == "left" else n
    _check_square("A", A, a_gpu, lda, order, side)
    _check_general("B", B, b_gpu, ldb, B.layout if b_gpu else layout, m, n)
    if not trmm:
        _check_general("C", C, c_gpu, ldc, C.layout if c_gpu else layout, m, n)
    return None


def _scratch(device, rows, cols, ld, layout, dtype):
    """A device temporary for the work this call queues: drawn from the handle's
    stream-ordered pool (``wg_buffer_alloc_async``) and returned to it in stream
    order on destroy(), so a call allocates and frees without mapping memory or
    waiting for the GPU."""
    outer = rows if layout == "row-major" else cols
    buf = nat.c_buf_p()
    nat.check(nat.lib.wg_buffer_alloc_async(device.handle, max(outer * ld, 1) * np.dtype(dtype).itemsize,
                                            ct.byref(buf)))
    return GpuMatrix(buf, rows, cols, ld, None, layout, device, dtype)


def _dense(device, order, dtype):
    return _scratch(device, order, order, order, "column-major", dtype)


def _symm(routine, device, side, uplo, m, n, alpha, A, lda, B, ldb, beta, C, ldc, layout):
    early = _validate_special(routine, device, side, uplo, None, None, m, n, alpha, A, lda, B, ldb, beta, C, ldc,
                              layout)
    if early is not None:
        return early
    f64 = routine.startswith("d")
    if f64 and alpha == 0 and beta == 1:
        # Reference BLAS quick return (src/dsymm/dsymm.mjs:143-145).
        return {} if isinstance(C, GpuMatrix) else {"C": C}
    gpu = isinstance(C, GpuMatrix)
    m, n, lda, ldb, ldc = (int(v) for v in (m, n, lda, ldb, ldc))
    order = m if side == "left" else n
    dt = np.float64 if f64 else np.float32
    scratch = []
    try:
        if gpu:
            GA, GB, GC = A, B, C
        else:
            GA = _upload(device, A, order, order, lda, layout)
            GB = _upload(device, B, m, n, ldb, layout)
            GC = _upload(device, C, m, n, ldc, layout)
            scratch += [GA, GB, GC]
        D = _dense(device, order, dt)
        scratch.append(D)
        # A = A^T, so a row-major A holds the other triangle in the column-major frame.
        lower = (uplo == "lower") == (GA.layout == "column-major")
        nat.check(nat.lib.wg_symmetrize(device.handle, np.dtype(dt).itemsize,
                                        nat.WG_UPLO_LOWER if lower else nat.WG_UPLO_UPPER, order, GA._buf, 0,
                                        GA.lda, D._buf, 0, order))
        if side == "left":
            r = _execute(f64, device, "no-transpose", "no-transpose", m, n, order, alpha, D, order, GB, ldb, beta,
                         GC, ldc, layout)
        else:
            r = _execute(f64, device, "no-transpose", "no-transpose", m, n, order, alpha, GB, ldb, D, order, beta,
                         GC, ldc, layout)
        if gpu:
            return r
        out = _download_into(GC, C)
        return {"C": out, **({"gpuTimeMs": r["gpuTimeMs"]} if "gpuTimeMs" in r else {})}
    finally:
        for G in scratch:
            G.destroy()


def _trmm(routine, device, side, uplo, transA, diag, m, n, alpha, A, lda, B, ldb, layout):
    early = _validate_special(routine, device, side, uplo, transA, diag, m, n, alpha, A, lda, B, ldb, None, None,
                              None, layout)
    if early is not None:
        return early
    f64 = routine.startswith("d")
    gpu = isinstance(B, GpuMatrix)
    m, n, lda, ldb = (int(v) for v in (m, n, lda, ldb))
    order = m if side == "left" else n
    dt = np.float64 if f64 else np.float32
    item = np.dtype(dt).itemsize
    scratch = []
    try:
        if gpu:
            GA, GB = A, B
        else:
            GA = _upload(device, A, order, order, lda, layout)
            GB = _upload(device, B, m, n, ldb, layout)
            scratch += [GA, GB]
        # A is not symmetric: a row-major A is A^T in the column-major frame, so
        # both the stored triangle and the transpose flip.
        cm = GA.layout == "column-major"
        lower = (uplo == "lower") == cm
        trans = (transA == "transpose") == cm
        D = _dense(device, order, dt)
        scratch.append(D)
        nat.check(nat.lib.wg_triangularize(device.handle, item, nat.WG_UPLO_LOWER if lower else nat.WG_UPLO_UPPER,
                                           int(trans), int(diag == "unit"), order, GA._buf, 0, GA.lda, D._buf, 0,
                                           order))
        # alpha*op(A)*B (or alpha*B*op(A)) into scratch with B's layout, then over B.
        outer = m if GB.layout == "row-major" else n
        T = _scratch(device, m, n, ldb, GB.layout, dt)
        scratch.append(T)
        X, Y = (D, GB) if side == "left" else (GB, D)
        r = _execute(f64, device, "no-transpose", "no-transpose", m, n, order, alpha, X, X.lda, Y, Y.lda, 0.0, T,
                     ldb, GB.layout)
        inner = n if GB.layout == "row-major" else m
        nat.check(nat.lib.wg_buffer_copy_2d(device.handle, T._buf, 0, ldb * item, GB._buf, 0, ldb * item, inner * item,
                                            outer))
        if gpu:
            nat.check(nat.lib.wg_device_sync(device.handle))
            return {"gpuTimeMs": r["gpuTimeMs"]} if "gpuTimeMs" in r else {}
        out = _download_into(GB, B)
        return {"B": out, **({"gpuTimeMs": r["gpuTimeMs"]} if "gpuTimeMs" in r else {})}
    finally:
        for G in scratch:
            G.destroy()


def ssymm(device, side, uplo, m, n, alpha, A, lda, B, ldb, beta, C, ldc, layout="row-major"):
    """C := alpha*A*B + beta*C (side 'left') or alpha*B*A + beta*C ('right'), A
    symmetric with its uplo triangle stored, in fp32 (src/ssymm/ssymm.mjs:29-44)."""
    return _symm("ssymm", device, side, uplo, m, n, alpha, A, lda, B, ldb, beta, C, ldc, layout)


def dsymm(device, side, uplo, m, n, alpha, A, lda, B, ldb, beta, C, ldc, layout="row-major"):
    """ssymm in native fp64 (src/dsymm/dsymm.mjs)."""
    return _symm("dsymm", device, side, uplo, m, n, alpha, A, lda, B, ldb, beta, C, ldc, layout)


def strmm(device, side, uplo, transA, diag, m, n, alpha, A, lda, B, ldb, layout="row-major"):
    """B := alpha*op(A)*B (side 'left') or alpha*B*op(A) ('right'), A triangular
    with its uplo triangle stored, in fp32 (src/strmm/strmm.mjs:25-48)."""
    return _trmm("strmm", device, side, uplo, transA, diag, m, n, alpha, A, lda, B, ldb, layout)


def dtrmm(device, side, uplo, transA, diag, m, n, alpha, A, lda, B, ldb, layout="row-major"):
    """strmm in native fp64 (src/dtrmm/dtrmm.mjs)."""
    return _trmm("dtrmm", device, side, uplo, transA, diag, m, n, alpha, A, lda, B, ldb, layout)


def _trsm(routine, device, side, uplo, transA, diag, m, n, alpha, A, lda, B, ldb, layout):
    early = _validate_special(routine, device, side, uplo, transA, diag, m, n, alpha, A, lda, B, ldb, None, None,
                              None, layout)
    if early is not None:
        return early
    gpu = isinstance(B, GpuMatrix)
    m, n, lda, ldb = (int(v) for v in (m, n, lda, ldb))
    order = m if side == "left" else n
    scratch = []
    try:
        if gpu:
            GA, GB = A, B
        else:
            GA = _upload(device, A, order, order, lda, layout)
            GB = _upload(device, B, m, n, ldb, layout)
            scratch += [GA, GB]
        # The column-major frame of B: a row-major B is B^T there, so the side
        # and m/n swap and the operator becomes op(A)^T. A row-major A is A^T
        # in that frame, which flips its stored triangle and once more the
        # transpose (src/strsm/strsm.mjs:244-257 flips both for the same reason).
        b_rm = GB.layout == "row-major"
        a_rm = GA.layout == "row-major"
        side_cm = (side == "left") != b_rm
        trans_cm = ((transA == "transpose") != b_rm) != a_rm
        lower_cm = (uplo == "lower") != a_rm
        mc, nc = (n, m) if b_rm else (m, n)
        ms = ct.c_float(0.0)
        nat.check(nat.lib.wg_strsm(device.handle, nat.WG_SIDE_LEFT if side_cm else nat.WG_SIDE_RIGHT,
                                   nat.WG_UPLO_LOWER if lower_cm else nat.WG_UPLO_UPPER, int(trans_cm),
                                   nat.WG_DIAG_UNIT if diag == "unit" else nat.WG_DIAG_NON_UNIT, mc, nc, float(alpha),
                                   GA._buf, 0, GA.lda, GB._buf, 0, GB.lda,
                                   ct.byref(ms) if device.benchmark else None))
        timed = {"gpuTimeMs": float(ms.value)} if device.benchmark else {}
        if gpu:
            nat.check(nat.lib.wg_device_sync(device.handle))
            return timed
        return {"B": _download_into(GB, B), **timed}
    finally:
        for G in scratch:
            G.destroy()


def strsm(device, side, uplo, transA, diag, m, n, alpha, A, lda, B, ldb, layout="row-major"):
    """Solves op(A)*X = alpha*B (side 'left') or X*op(A) = alpha*B ('right') for X,
    A triangular with its uplo triangle stored, overwriting B, in fp32
    (src/strsm/strsm.mjs:160-583). Plain arrays come back as a new array
    (``{"B": X}``); a GpuMatrix B is solved in place. alpha = 0 makes B a literal
    zero without reading A or B. Infinity and NaN land where substitution puts
    them (tests/strsm/src/test.strsm.js:498-578), for GpuMatrix operands too."""
    return _trsm("strsm", device, side, uplo, transA, diag, m, n, alpha, A, lda, B, ldb, layout)
