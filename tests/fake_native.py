"""A CPU stand-in for libwgblas_b200.so, for tests of the Python layer only.

Implements, in numpy, the column-major-frame semantics that include/wgblas.h
documents for the entry points the Python wrappers call: buffers are host
byte arrays, GEMM / gemmtr / symmetrize / triangularize / strsm / gemv compute
in float64 and store in the buffer's type. It checks argument plumbing (the
row-major to column-major mapping of layouts, sides, triangles and
transposes, offsets, leading dimensions, strides and return shapes), not
kernel arithmetic; host-only entry points (the random generators) are taken
from the real library.
"""
from __future__ import annotations

import ctypes as ct

import numpy as np

HOST_ONLY = ("wg_random_f32", "wg_random_f64", "wg_random_normal_f32", "wg_random_normal_f64", "wg_last_error")
LOWER, UPPER = 1, 2


class FakeLib:
    def __init__(self, real):
        self._real = real
        self.bufs = {}
        self._next = 4096
        self.calls = []

    def __getattr__(self, name):
        if name in HOST_ONLY:
            return getattr(self._real, name)
        raise AttributeError(f"the fake library has no {name}")

    # ---- devices (init / cleanup / gpuName tests) ----------------------------

    n_devices = 2
    opened = 0
    closed = 0

    def wg_device_count(self, ref):
        ref._obj.value = self.n_devices
        return 0

    def wg_device_open(self, ordinal, flags, ref):
        self._next += 16
        ref._obj.value = self._next
        self.opened += 1
        return 0

    def wg_device_close(self, dev):
        self.closed += 1
        return 0

    def wg_device_name(self, dev, buf, size):
        ct.memmove(buf, b"Fake B200\0", 10)
        return 0

    def wg_device_props_get(self, dev, ref):
        p = ref._obj
        p.ordinal, p.sm_count, p.cc_major, p.cc_minor, p.total_mem, p.flags = 0, 148, 10, 0, 183 << 30, 0
        return 0

    # ---- buffers -------------------------------------------------------------

    def _key(self, b):
        return b if isinstance(b, int) else b.value

    def _view(self, b, dt, off=0):
        return np.frombuffer(self.bufs[self._key(b)], dt)[off:]

    def wg_buffer_alloc(self, dev, nbytes, ref):
        self._next += 16
        self.bufs[self._next] = bytearray(int(nbytes))
        ref._obj.value = self._next
        return 0

    def wg_buffer_alloc_async(self, dev, nbytes, ref):
        return self.wg_buffer_alloc(dev, nbytes, ref)

    def wg_buffer_free(self, b):
        self.bufs.pop(self._key(b), None)
        return 0

    def wg_buffer_upload(self, b, off, ptr, nbytes):
        self.bufs[self._key(b)][off:off + nbytes] = ct.string_at(ptr, nbytes)
        return 0

    def wg_buffer_download(self, b, off, ptr, nbytes):
        ct.memmove(ptr, bytes(self.bufs[self._key(b)][off:off + nbytes]), nbytes)
        return 0

    def wg_buffer_download_2d(self, b, off, spitch, ptr, dpitch, width, rows):
        src = self.bufs[self._key(b)]
        base = ptr.value if isinstance(ptr, ct.c_void_p) else ptr
        for r in range(rows):
            ct.memmove(base + r * dpitch, bytes(src[off + r * spitch: off + r * spitch + width]), width)
        return 0

    def wg_buffer_copy_2d(self, dev, src, soff, spitch, dst, doff, dpitch, width, rows):
        s, d = self.bufs[self._key(src)], self.bufs[self._key(dst)]
        for r in range(rows):
            d[doff + r * dpitch: doff + r * dpitch + width] = s[soff + r * spitch: soff + r * spitch + width]
        return 0

    def wg_device_sync(self, dev):
        return 0

    def wg_device_check(self, dev):
        return 0

    # ---- column-major helpers ------------------------------------------------

    @staticmethod
    def _mat(buf, ld, rows, cols):
        """The rows x cols column-major matrix at the start of `buf`, as float64."""
        if rows == 0 or cols == 0:
            return np.zeros((rows, cols))
        idx = np.arange(rows)[:, None] + np.arange(cols)[None, :] * ld
        return buf[idx].astype(np.float64)

    @staticmethod
    def _store(buf, ld, val, mask=None):
        rows, cols = val.shape
        idx = np.arange(rows)[:, None] + np.arange(cols)[None, :] * ld
        if mask is None:
            buf[idx] = val.astype(buf.dtype)
        else:
            buf[idx[mask]] = val[mask].astype(buf.dtype)

    def _gemm(self, dt, uplo, tA, tB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc):
        self.calls.append(("gemm", dt, uplo, tA, tB, m, n, k))
        if m == 0 or n == 0:
            return 0
        if alpha != 0 and k > 0:
            opA = self._mat(A, lda, k, m).T if tA else self._mat(A, lda, m, k)
            opB = self._mat(B, ldb, n, k).T if tB else self._mat(B, ldb, k, n)
            res = float(alpha) * (opA @ opB)
        else:
            res = np.zeros((m, n))
        if beta != 0:
            res = res + float(beta) * self._mat(C, ldc, m, n)
        mask = None
        if uplo in (LOWER, UPPER):
            i, j = np.meshgrid(np.arange(m), np.arange(n), indexing="ij")
            mask = (j <= i) if uplo == LOWER else (j >= i)
        self._store(C, ldc, res, mask)
        return 0

    def _dev(self, dt, *a):
        # (dev, [uplo], tA, tB, m, n, k, alpha, A, offA, lda, B, offB, ldb, beta, C, offC, ldc, ms)
        uplo, a = (a[1], a[2:]) if len(a) == 19 else (0, a[1:])
        tA, tB, m, n, k, alpha, A, oA, lda, B, oB, ldb, beta, C, oC, ldc, _ = a
        return self._gemm(dt, uplo, tA, tB, m, n, k, alpha, self._view(A, dt, oA), lda, self._view(B, dt, oB), ldb,
                          beta, self._view(C, dt, oC), ldc)

    def _host(self, dt, *a):
        # (dev, [uplo], tA, tB, m, n, k, alpha, A, lda, B, ldb, beta, C_in, C_out, ldc, ms)
        uplo, a = (a[1], a[2:]) if len(a) == 17 else (0, a[1:])
        tA, tB, m, n, k, alpha, A, lda, B, ldb, beta, Cin, Cout, ldc, _ = a
        item = np.dtype(dt).itemsize

        def arr(ptr, count):
            if count <= 0:
                return np.zeros(0, dt)
            return np.frombuffer((ct.c_char * (count * item)).from_address(ptr.value), dt).copy()

        ra, ca = (k, m) if tA else (m, k)
        rb, cb = (n, k) if tB else (k, n)
        Av = arr(A, (ca - 1) * lda + ra) if alpha != 0 and k > 0 else np.zeros(0, dt)
        Bv = arr(B, (cb - 1) * ldb + rb) if alpha != 0 and k > 0 else np.zeros(0, dt)
        cnt = (n - 1) * ldc + m if m and n else 0
        Cv = arr(Cin, cnt)
        out = arr(Cout, cnt)
        self._gemm(dt, uplo, tA, tB, m, n, k, alpha, Av, lda, Bv, ldb, beta, Cv, ldc)
        i, j = np.meshgrid(np.arange(m), np.arange(n), indexing="ij")
        idx = (i + j * ldc).ravel()
        out[idx] = Cv[idx]
        if cnt:
            ct.memmove(Cout.value, out.tobytes(), cnt * item)
        return 0

    def wg_sgemm(self, *a):
        return self._dev(np.float32, *a)

    def wg_dgemm(self, *a):
        return self._dev(np.float64, *a)

    def wg_sgemmtr(self, *a):
        return self._dev(np.float32, *a)

    def wg_dgemmtr(self, *a):
        return self._dev(np.float64, *a)

    def wg_sgemm_host(self, *a):
        return self._host(np.float32, *a)

    def wg_dgemm_host(self, *a):
        return self._host(np.float64, *a)

    def wg_sgemmtr_host(self, *a):
        return self._host(np.float32, *a)

    def wg_dgemmtr_host(self, *a):
        return self._host(np.float64, *a)

    # ---- operand passes, strsm, gemv ----------------------------------------

    def wg_symmetrize(self, dev, elem, uplo, n, A, oA, lda, out, oO, ldo):
        dt = np.float32 if elem == 4 else np.float64
        M = self._mat(self._view(A, dt, oA), lda, n, n)
        low = np.tril(M) if uplo == LOWER else np.triu(M)
        full = low + low.T - np.diag(np.diag(M))
        self._store(self._view(out, dt, oO), ldo, full)
        return 0

    def wg_triangularize(self, dev, elem, uplo, trans, unit, n, A, oA, lda, out, oO, ldo):
        dt = np.float32 if elem == 4 else np.float64
        M = self._mat(self._view(A, dt, oA), lda, n, n)
        T = np.tril(M, -1) if uplo == LOWER else np.triu(M, 1)
        T = T + (np.eye(n) if unit else np.diag(np.diag(M)))
        self._store(self._view(out, dt, oO), ldo, T.T if trans else T)
        return 0

    def wg_strsm(self, dev, side, uplo, trans, diag, m, n, alpha, A, oA, lda, B, oB, ldb, ms):
        self.calls.append(("strsm", side, uplo, trans, diag, m, n))
        if m == 0 or n == 0:
            return 0
        Bb = self._view(B, np.float32, oB)
        if alpha == 0:
            self._store(Bb, ldb, np.zeros((m, n)))
            return 0
        order = m if side == 0 else n
        M = self._mat(self._view(A, np.float32, oA), lda, order, order)
        T = np.tril(M, -1) if uplo == LOWER else np.triu(M, 1)
        T = T + (np.eye(order) if diag else np.diag(np.diag(M)))
        op = T.T if trans else T
        X = float(alpha) * self._mat(Bb, ldb, m, n)
        sol = np.linalg.solve(op, X) if side == 0 else np.linalg.solve(op.T, X.T).T
        self._store(Bb, ldb, sol)
        return 0

    def _gemv(self, dt, dev, trans, m, n, alpha, A, oA, lda, x, ox, incx, beta, y, oy, incy, ms):
        self.calls.append(("gemv", dt, trans, m, n))
        if m == 0 or n == 0 or (alpha == 0 and beta == 1):
            return 0
        xlen, ylen = (m, n) if trans else (n, m)
        yv = self._view(y, dt, oy)
        iy = np.arange(ylen) * incy
        res = np.zeros(ylen)
        if alpha != 0:
            M = self._mat(self._view(A, dt, oA), lda, m, n)
            xv = self._view(x, dt, ox)[np.arange(xlen) * incx].astype(np.float64)
            res = float(alpha) * ((M.T if trans else M) @ xv)
        if beta != 0:
            res = res + float(beta) * yv[iy].astype(np.float64)
        yv[iy] = res.astype(dt)
        return 0

    def wg_sgemv(self, *a):
        return self._gemv(np.float32, *a)

    def wg_dgemv(self, *a):
        return self._gemv(np.float64, *a)
