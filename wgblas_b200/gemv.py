"""``sgemv`` / ``dgemv`` with wgblas's arguments: y := alpha*op(A)*x + beta*y.

Mirrors src/sgemv/sgemv.mjs:19-254 and src/dgemv/dgemv.mjs: the same argument
order, validation order and messages, and return shapes. Typed arrays come
back as a new ``{"y": ...}`` (strided gaps of y keep their values); a
GpuMatrix A with GpuVector x and y updates y in place and returns ``{}`` (plus
``gpuTimeMs`` on a benchmark device). m or n = 0 returns y as it is; dgemv keeps
the reference BLAS quick return for alpha = 0 with beta = 1
(src/dgemv/dgemv.mjs), returning the very array it was given.

The work is one call of ``wg_sgemv`` / ``wg_dgemv`` in the column-major frame. A
row-major A (m x n, lda >= n) is A^T there, so the transpose flips and m, n
swap, as the reference swaps into its row-major kernel frame for a
column-major A (src/sgemv/sgemv.mjs:94-100). dgemv computes in native fp64.
"""
from __future__ import annotations

import ctypes as ct
import math

import numpy as np

from . import _native as nat
from ._runtime import Error, require_gpu_device, require_same_device
from .classes import GpuMatrix, GpuVector, _is_int, is_f32_array, is_f64_array
from .gemm import _LAYOUTS, _TRANS, _is_number


def _check_scalar(name, v):
    if not _is_number(v):
        raise Error(f"{name} must be a number.")
    if math.isnan(v):
        raise Error(f"{name} must not be NaN.")
    if not math.isfinite(v):
        raise Error(f"{name} must be finite.")


def _length(v):
    return v.length if isinstance(v, GpuVector) else v.size


def _validate(routine, device, trans, m, n, alpha, A, lda, x, incx, beta, y, incy, layout):
    """src/sgemv/sgemv.mjs:33-116 (src/dgemv/dgemv.mjs adds the dtype checks).
    Returns (quick_return_value | None, kernel-frame dims)."""
    f64 = routine == "dgemv"
    arr = "Float64Array" if f64 else "Float32Array"
    is_arr = is_f64_array if f64 else is_f32_array
    a_gpu, x_gpu, y_gpu = isinstance(A, GpuMatrix), isinstance(x, GpuVector), isinstance(y, GpuVector)
    require_gpu_device(device)
    require_same_device(device, routine, {"A": A, "x": x, "y": y})
    if trans not in _TRANS:
        raise Error("trans must be 'no-transpose' or 'transpose'.")
    if layout not in _LAYOUTS:
        raise Error("layout must be 'row-major' or 'column-major'.")
    _check_scalar("alpha", alpha)
    _check_scalar("beta", beta)
    if not all(_is_int(v) for v in (m, n, incx, incy, lda)):
        raise Error("m, n, incx, incy, and lda must be integers.")
    if incx <= 0 or incy <= 0:
        raise Error("incx and incy must be positive.")
    if not a_gpu and not is_arr(A):
        raise Error(f"A must be a {arr} or GpuMatrix.")
    if f64 and a_gpu and A.dtype is not np.float64:
        raise Error("A must be a Float64Array-backed GpuMatrix.")
    if not x_gpu and not is_arr(x):
        raise Error(f"x must be a {arr} or GpuVector.")
    if not y_gpu and not is_arr(y):
        raise Error(f"y must be a {arr} or GpuVector.")
    if f64 and x_gpu and x.dtype is not np.float64:
        raise Error("x must be a Float64Array-backed GpuVector.")
    if f64 and y_gpu and y.dtype is not np.float64:
        raise Error("y must be a Float64Array-backed GpuVector.")
    if x_gpu != y_gpu:
        raise Error(f"x and y must be the same type (both {arr} or both GpuVector).")
    if x_gpu and not a_gpu:
        raise Error("A must be a GpuMatrix when x and y are GpuVectors.")
    if a_gpu and not x_gpu:
        raise Error("x and y must be GpuVectors when A is a GpuMatrix.")
    if x_gpu and x._buf is y._buf:
        raise Error("x and y must not reference the same GPU buffer when both are GpuVectors.")
    if a_gpu and y_gpu and A._buf is y._buf:
        raise Error("A and y must not reference the same GPU buffer.")
    if a_gpu and lda != A.lda:
        raise Error("lda must match A.lda when A is a GpuMatrix.")
    if a_gpu and (A.rows < m or A.cols < n):
        raise Error("A is too small for the given m and n.")
    if m < 0 or n < 0:
        raise Error("m and n must be non-negative.")
    if m == 0 or n == 0:
        return ({} if y_gpu else {"y": y}), None
    # The reference's row-major kernel frame (sgemv.mjs:94-100).
    eff = A.layout if a_gpu else layout
    km, kn, ktrans = (n, m, "transpose" if trans == "no-transpose" else "no-transpose") \
        if eff == "column-major" else (m, n, trans)
    no_t = ktrans == "no-transpose"
    x_len, y_len = (kn, km) if no_t else (km, kn)
    if lda < kn:
        raise Error("lda must be >= n.")
    if not a_gpu and A.size < (km - 1) * lda + kn:
        raise Error("A does not have enough elements for the given m, n, and lda.")
    if _length(x) < (x_len - 1) * incx + 1:
        raise Error("x does not have enough elements for the given dimensions and incx.")
    if _length(y) < (y_len - 1) * incy + 1:
        raise Error("y does not have enough elements for the given dimensions and incy.")
    if f64 and alpha == 0 and beta == 1:
        return ({} if y_gpu else {"y": y}), None
    return None, (km, kn, no_t, x_len, y_len)


def _scratch(device, arr, count):
    """A device buffer holding the first `count` elements of a plain array."""
    buf = nat.c_buf_p()
    nbytes = max(count, 1) * arr.itemsize
    nat.check(nat.lib.wg_buffer_alloc(device.handle, nbytes, ct.byref(buf)))
    try:
        if count:
            nat.check(nat.lib.wg_buffer_upload(buf, 0, arr.ctypes.data_as(ct.c_void_p), count * arr.itemsize))
    except Exception:
        nat.lib.wg_buffer_free(buf)
        raise
    return buf


def _gemv(routine, device, trans, m, n, alpha, A, lda, x, incx, beta, y, incy, layout):
    early, dims = _validate(routine, device, trans, m, n, alpha, A, lda, x, incx, beta, y, incy, layout)
    if early is not None:
        return early
    km, kn, no_t, x_len, y_len = dims
    f64 = routine == "dgemv"
    fn = nat.lib.wg_dgemv if f64 else nat.lib.wg_sgemv
    # Row-major kernel frame (km x kn, row stride lda) = column-major kn x km:
    # its no-transpose is the column-major transpose.
    cm_trans = 1 if no_t else 0
    ms = ct.c_float(0.0)
    ms_p = ct.byref(ms) if device.benchmark else None
    if isinstance(y, GpuVector):
        nat.check(fn(device.handle, cm_trans, int(kn), int(km), float(alpha), A._buf, 0, int(lda), x._buf, 0, int(incx),
                     float(beta), y._buf, 0, int(incy), ms_p))
        if not device.benchmark:
            nat.check(nat.lib.wg_device_sync(device.handle))
            return {}
        return {"gpuTimeMs": float(ms.value)}
    a_count = (km - 1) * lda + kn
    x_count = (x_len - 1) * incx + 1
    y_count = (y_len - 1) * incy + 1
    bufs = []
    try:
        bufs.append(_scratch(device, np.ascontiguousarray(A), a_count))
        bufs.append(_scratch(device, np.ascontiguousarray(x), x_count))
        bufs.append(_scratch(device, np.ascontiguousarray(y), y_count))
        nat.check(fn(device.handle, cm_trans, int(kn), int(km), float(alpha), bufs[0], 0, int(lda), bufs[1], 0,
                     int(incx), float(beta), bufs[2], 0, int(incy), ms_p))
        out = y.copy()
        nat.check(nat.lib.wg_buffer_download(bufs[2], 0, out.ctypes.data_as(ct.c_void_p), y_count * out.itemsize))
    finally:
        for b in bufs:
            nat.lib.wg_buffer_free(b)
    return {"y": out, "gpuTimeMs": float(ms.value)} if device.benchmark else {"y": out}


def sgemv(device, trans, m, n, alpha, A, lda, x, incx, beta, y, incy, layout="row-major"):
    """y := alpha*op(A)*x + beta*y in fp32 (src/sgemv/sgemv.mjs:19-254)."""
    return _gemv("sgemv", device, trans, m, n, alpha, A, lda, x, incx, beta, y, incy, layout)


def dgemv(device, trans, m, n, alpha, A, lda, x, incx, beta, y, incy, layout="row-major"):
    """y := alpha*op(A)*x + beta*y in native fp64 (src/dgemv/dgemv.mjs)."""
    return _gemv("dgemv", device, trans, m, n, alpha, A, lda, x, incx, beta, y, incy, layout)
