"""Resident operands: ``GpuMatrix`` and ``GpuVector`` on cudaMalloc'd buffers.

Mirrors src/classes/GpuMatrix.mjs:13-207 and src/classes/GpuVector.mjs:13-106.
Differences by design: an f64 matrix is stored as native doubles (the
reference keeps a double-double hi/lo pair of f32 buffers), so ``_loBuf`` is
always None and ``read()`` returns the stored doubles exactly. Complex data is
outside the GEMM path and is not accepted.

``Float32Array`` / ``Float64Array`` stand for the JS typed arrays: 1-D numpy
arrays of float32 / float64.
"""
from __future__ import annotations

import ctypes as ct

import numpy as np

from . import _native as nat
from ._runtime import Device, Error, getDevice


def Float32Array(x) -> np.ndarray:
    """A 1-D float32 array: ``Float32Array(n)`` is n zeros, ``Float32Array(seq)`` copies."""
    if isinstance(x, (int, np.integer)) and not isinstance(x, bool):
        return np.zeros(int(x), np.float32)
    return np.array(x, dtype=np.float32).reshape(-1)


def Float64Array(x) -> np.ndarray:
    if isinstance(x, (int, np.integer)) and not isinstance(x, bool):
        return np.zeros(int(x), np.float64)
    return np.array(x, dtype=np.float64).reshape(-1)


def is_f32_array(x) -> bool:
    return isinstance(x, np.ndarray) and x.dtype == np.float32 and x.ndim == 1


def is_f64_array(x) -> bool:
    return isinstance(x, np.ndarray) and x.dtype == np.float64 and x.ndim == 1


class _Pinned:
    """Owner of a page-locked host allocation; freed when the last view dies."""

    def __init__(self, nbytes: int):
        p = ct.c_void_p()
        nat.check(nat.lib.wg_host_alloc(max(nbytes, 1), ct.byref(p)))
        self.ptr = p.value
        # Held here so the array can still be freed while the interpreter shuts
        # down and module globals are already cleared.
        self._free = nat.lib.wg_host_free

    def __del__(self):
        if getattr(self, "ptr", None):
            self._free(ct.c_void_p(self.ptr))
            self.ptr = None


def pinned_empty(n: int, dtype=np.float32) -> np.ndarray:
    """An uninitialised 1-D array in page-locked host memory: host<->device copies
    of it run asynchronously at full PCIe rate. The allocation lives as long as
    any view of the array."""
    dtype = np.dtype(dtype)
    nbytes = max(n * dtype.itemsize, 1)
    owner = _Pinned(nbytes)
    buf = (ct.c_char * nbytes).from_address(owner.ptr)
    buf._owner = owner  # ctypes instances accept attributes; numpy keeps `buf` as base
    return np.frombuffer(buf, dtype=dtype, count=n)


def _alloc(device: Device, nbytes: int):
    h = nat.c_buf_p()
    nat.check(nat.lib.wg_buffer_alloc(device.handle, nbytes, ct.byref(h)))
    return h


def _upload(buf, arr: np.ndarray) -> None:
    arr = np.ascontiguousarray(arr)
    nat.check(nat.lib.wg_buffer_upload(buf, 0, arr.ctypes.data_as(ct.c_void_p), arr.nbytes))


class GpuMatrix:
    """A matrix resident in device memory (src/classes/GpuMatrix.mjs:13-33)."""

    def __init__(self, buffer, rows, cols, lda, loBuffer=None, layout="row-major", device=None,
                 dtype=np.float32):
        self._buf = buffer
        self._loBuf = loBuffer
        self.rows = rows
        self.cols = cols
        self.lda = lda
        self.layout = layout
        self.dtype = np.dtype(dtype).type
        self.device = device if device is not None else getDevice()

    @staticmethod
    def from_(device_or_data, *rest) -> "GpuMatrix":
        """``GpuMatrix.from([device,] data, rows, cols, lda?, layout?)``
        (src/classes/GpuMatrix.mjs:43-140): validates and uploads ``outer*lda``
        elements (outer = rows for row-major, cols for column-major)."""
        explicit = isinstance(device_or_data, Device)
        device = device_or_data if explicit else getDevice()
        rest = list(rest)
        data = rest.pop(0) if explicit else device_or_data
        rows = rest[0] if len(rest) > 0 else None
        cols = rest[1] if len(rest) > 1 else None
        lda = rest[2] if len(rest) > 2 else None
        layout = rest[3] if len(rest) > 3 and rest[3] is not None else "row-major"
        if layout not in ("row-major", "column-major"):
            raise Error("layout must be 'row-major' or 'column-major'.")
        is_row = layout == "row-major"
        if lda is None:
            lda = cols if is_row else rows
        if not (is_f32_array(data) or is_f64_array(data)):
            raise Error("GpuMatrix.from expects a Float32Array, Float64Array, Complex32Array, "
                        "or Complex64Array.")
        if not _is_int(rows) or rows <= 0:
            raise Error("rows must be a positive integer.")
        if not _is_int(cols) or cols <= 0:
            raise Error("cols must be a positive integer.")
        min_lda = cols if is_row else rows
        if not _is_int(lda) or lda < min_lda:
            raise Error(f"lda must be an integer >= {'cols' if is_row else 'rows'}.")
        rows, cols, lda = int(rows), int(cols), int(lda)
        outer = rows if is_row else cols
        if data.size < outer * lda:
            raise Error("data does not have enough elements for the given rows, cols, and lda.")
        src = data[: outer * lda]
        buf = _alloc(device, src.nbytes)
        try:
            _upload(buf, src)
        except Exception:
            nat.lib.wg_buffer_free(buf)
            raise
        return GpuMatrix(buf, rows, cols, lda, None, layout, device, data.dtype)

    def read(self, out: np.ndarray | None = None) -> np.ndarray:
        """The matrix as a dense 1-D array in its own layout, lda padding stripped
        (src/classes/GpuMatrix.mjs:142-202). ``out`` (an addition) receives the
        values instead of a new array, e.g. a page-locked one from
        ``pinned_empty`` for a full-rate copy."""
        self._require_live()
        is_row = self.layout != "column-major"
        outer = self.rows if is_row else self.cols
        inner = self.cols if is_row else self.rows
        item = np.dtype(self.dtype).itemsize
        if out is None:
            out = np.empty(outer * inner, self.dtype)
        elif (out.dtype != np.dtype(self.dtype) or out.size != outer * inner or out.ndim != 1
              or not out.flags.c_contiguous):
            raise Error("out must be a contiguous 1-D array of the matrix's dtype and rows*cols elements.")
        nat.check(nat.lib.wg_buffer_download_2d(self._buf, 0, self.lda * item,
                                                out.ctypes.data_as(ct.c_void_p), inner * item,
                                                inner * item, outer))
        return out

    def write(self, data: np.ndarray) -> None:
        """Copies ``data`` (the outer*lda elements ``from`` would take, same dtype)
        into the matrix's buffer (an addition: refills a resident matrix without
        a new allocation)."""
        self._require_live()
        outer = self.rows if self.layout != "column-major" else self.cols
        data = np.asarray(data)
        if data.dtype != np.dtype(self.dtype) or data.size < outer * self.lda:
            raise Error("data must have the matrix's dtype and at least outer*lda elements.")
        _upload(self._buf, data.reshape(-1)[: outer * self.lda])

    def destroy(self) -> None:
        if self._buf is not None:
            nat.lib.wg_buffer_free(self._buf)
            self._buf = None

    def device_ptr(self) -> int:
        self._require_live()
        p = ct.c_void_p()
        nat.check(nat.lib.wg_buffer_device_ptr(self._buf, ct.byref(p)))
        return p.value or 0

    def _require_live(self):
        if self._buf is None:
            raise Error("GpuMatrix has been destroyed.")

    def __repr__(self):
        return (f"<GpuMatrix {self.rows}x{self.cols} lda={self.lda} {self.layout} "
                f"{np.dtype(self.dtype).name} on {self.device!r}>")


def _gpu_matrix_empty(device: Device, rows: int, cols: int, lda: int | None = None,
                      layout: str = "row-major", dtype=np.float32) -> GpuMatrix:
    """An uninitialised resident matrix (no upload) — for benchmarks and outputs."""
    is_row = layout == "row-major"
    lda = (cols if is_row else rows) if lda is None else lda
    outer = rows if is_row else cols
    buf = _alloc(device, outer * lda * np.dtype(dtype).itemsize)
    return GpuMatrix(buf, rows, cols, lda, None, layout, device, dtype)


GpuMatrix.empty = staticmethod(_gpu_matrix_empty)
setattr(GpuMatrix, "from", GpuMatrix.from_)


class GpuVector:
    """A vector resident in device memory (src/classes/GpuVector.mjs:13-106)."""

    def __init__(self, buffer, length, dtype=np.float32, loBuffer=None, device=None):
        self._buf = buffer
        self._loBuf = loBuffer
        self.length = length
        self.dtype = np.dtype(dtype).type
        self.device = device if device is not None else getDevice()

    @staticmethod
    def from_(device_or_data, maybe_data=None) -> "GpuVector":
        explicit = isinstance(device_or_data, Device)
        device = device_or_data if explicit else getDevice()
        data = maybe_data if explicit else device_or_data
        if not (is_f32_array(data) or is_f64_array(data)):
            raise Error("GpuVector.from expects a Float32Array, Float64Array, Complex32Array, "
                        "or Complex64Array.")
        buf = _alloc(device, data.nbytes)
        try:
            _upload(buf, data)
        except Exception:
            nat.lib.wg_buffer_free(buf)
            raise
        return GpuVector(buf, data.size, data.dtype, None, device)

    def read(self) -> np.ndarray:
        if self._buf is None:
            raise Error("GpuVector has been destroyed.")
        out = np.empty(self.length, self.dtype)
        nat.check(nat.lib.wg_buffer_download(self._buf, 0, out.ctypes.data_as(ct.c_void_p), out.nbytes))
        return out

    def destroy(self) -> None:
        if self._buf is not None:
            nat.lib.wg_buffer_free(self._buf)
            self._buf = None


setattr(GpuVector, "from", GpuVector.from_)


def _is_int(x) -> bool:
    """Number.isInteger: an int (not bool) or an integral finite float."""
    if isinstance(x, bool):
        return False
    if isinstance(x, (int, np.integer)):
        return True
    if isinstance(x, (float, np.floating)):
        return bool(np.isfinite(x)) and float(x).is_integer()
    return False
