"""The Python layer over a CPU stand-in of the C ABI (tests/fake_native.py): every
public routine, through host arrays and GpuMatrix/GpuVector operands in any mix
of layouts, must hand the library a column-major call whose result, read back
in the caller's own layout, equals the routine's definition computed directly
in that layout. This checks the layout, side, triangle and transpose mapping,
offsets, leading dimensions, strides, padding and return shapes without a GPU;
the kernels' arithmetic is checked on the GPU. CPU only."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import bits_equal
from fake_native import FakeLib

LAYOUTS = ("row-major", "column-major")
TRANS = ("no-transpose", "transpose")


@pytest.fixture()
def env(wg, monkeypatch):
    from wgblas_b200 import _native as nat

    fake = FakeLib(nat.lib)
    monkeypatch.setattr(nat, "lib", fake)
    dev = wg.Device(object(), 0, False, {}, "fake")
    return wg, dev, fake


def stored(rows, cols, layout, pad, rng, dt=np.float32):
    """A rows x cols matrix stored in `layout` with ld = inner + pad: (array, ld)."""
    ld = (cols if layout == "row-major" else rows) + pad
    outer = rows if layout == "row-major" else cols
    return (rng.random(outer * ld) * 2 - 1).astype(dt), ld


def mat(X, ld, rows, cols, layout):
    i = np.arange(rows)[:, None]
    j = np.arange(cols)[None, :]
    idx = (i * ld + j) if layout == "row-major" else (j * ld + i)
    return X[idx].astype(np.float64), idx


def check_block(got, src, idx, want, mask=None, rtol=2e-5):
    """`want` at idx (only where mask), everything else in got bit-identical to src."""
    keep = np.ones(got.size, bool)
    sel = idx if mask is None else idx[mask]
    keep[sel.ravel()] = False
    assert bits_equal(got[keep], src[keep]), "an element outside the result changed"
    w = want if mask is None else want[mask]
    assert np.allclose(got[sel].astype(np.float64), w, rtol=rtol, atol=rtol)


def op(M, t):
    return M.T if t == "transpose" else M


@pytest.mark.parametrize("layout", LAYOUTS)
@pytest.mark.parametrize("tA", TRANS)
@pytest.mark.parametrize("tB", TRANS)
@pytest.mark.parametrize("routine", ["sgemm", "dgemm"])
def test_gemm_host_arrays(env, layout, tA, tB, routine):
    wg, dev, _ = env
    dt = np.float64 if routine == "dgemm" else np.float32
    rng = np.random.default_rng(1)
    m, n, k = 7, 5, 4
    A, lda = stored(*((m, k) if tA == "no-transpose" else (k, m)), layout, 2, rng, dt)
    B, ldb = stored(*((k, n) if tB == "no-transpose" else (n, k)), layout, 1, rng, dt)
    C, ldc = stored(m, n, layout, 3, rng, dt)
    got = getattr(wg, routine)(dev, tA, tB, m, n, k, 0.75, A, lda, B, ldb, -0.5, C, ldc, layout)["C"]
    Am, _ = mat(A, lda, *((m, k) if tA == "no-transpose" else (k, m)), layout)
    Bm, _ = mat(B, ldb, *((k, n) if tB == "no-transpose" else (n, k)), layout)
    Cm, idx = mat(C, ldc, m, n, layout)
    check_block(got, C, idx, 0.75 * op(Am, tA) @ op(Bm, tB) - 0.5 * Cm)


@pytest.mark.parametrize("la,lb,lc", [("row-major", "column-major", "row-major"),
                                      ("column-major", "row-major", "column-major"),
                                      ("column-major", "column-major", "row-major")])
def test_gemm_gpu_matrices_with_mixed_layouts(env, la, lb, lc):
    wg, dev, _ = env
    rng = np.random.default_rng(2)
    m, n, k = 6, 9, 5
    A, lda = stored(m, k, la, 1, rng)
    B, ldb = stored(n, k, lb, 0, rng)
    C, ldc = stored(m, n, lc, 2, rng)
    GA = wg.GpuMatrix.from_(dev, A, m, k, lda, la)
    GB = wg.GpuMatrix.from_(dev, B, n, k, ldb, lb)
    GC = wg.GpuMatrix.from_(dev, C, m, n, ldc, lc)
    assert wg.sgemm(dev, "no-transpose", "transpose", m, n, k, 1.5, GA, lda, GB, ldb, 0.25, GC, ldc) == {}
    got = GC.read()
    Am, _ = mat(A, lda, m, k, la)
    Bm, _ = mat(B, ldb, n, k, lb)
    Cm, _ = mat(C, ldc, m, n, lc)
    want = 1.5 * Am @ Bm.T + 0.25 * Cm
    assert np.allclose(got.reshape((m, n) if lc == "row-major" else (n, m)),
                       want if lc == "row-major" else want.T, rtol=2e-5, atol=2e-5)


@pytest.mark.parametrize("layout", LAYOUTS)
@pytest.mark.parametrize("uplo", ["lower", "upper"])
@pytest.mark.parametrize("routine", ["sgemmtr", "ssyrk", "ssyr2k", "dsyrk"])
def test_gemmtr_family_writes_the_named_triangle(env, layout, uplo, routine):
    wg, dev, _ = env
    dt = np.float64 if routine.startswith("d") else np.float32
    rng = np.random.default_rng(3)
    n, k = 6, 4
    i, j = np.meshgrid(np.arange(n), np.arange(n), indexing="ij")
    tri = (j <= i) if uplo == "lower" else (j >= i)
    C, ldc = stored(n, n, layout, 2, rng, dt)
    Cm, idx = mat(C, ldc, n, n, layout)
    fn = getattr(wg, routine)
    if routine == "sgemmtr":
        A, lda = stored(n, k, layout, 1, rng, dt)
        B, ldb = stored(k, n, layout, 1, rng, dt)
        got = fn(dev, uplo, "no-transpose", "no-transpose", n, n, k, 0.5, A, lda, B, ldb, 2.0, C, ldc, layout)["C"]
        want = 0.5 * mat(A, lda, n, k, layout)[0] @ mat(B, ldb, k, n, layout)[0] + 2.0 * Cm
    else:
        A, lda = stored(k, n, layout, 1, rng, dt)  # trans = 'transpose': op(A) = A^T is n x k
        Am = mat(A, lda, k, n, layout)[0].T
        if routine.endswith("syrk"):
            got = fn(dev, uplo, "transpose", n, k, 0.5, A, lda, 2.0, C, ldc, layout)["C"]
            want = 0.5 * Am @ Am.T + 2.0 * Cm
        else:
            B, ldb = stored(k, n, layout, 0, rng, dt)
            Bm = mat(B, ldb, k, n, layout)[0].T
            got = fn(dev, uplo, "transpose", n, k, 0.5, A, lda, B, ldb, 2.0, C, ldc, layout)["C"]
            want = 0.5 * (Am @ Bm.T + Bm @ Am.T) + 2.0 * Cm
    check_block(got, C, idx, want, tri)


def tri_of(Am, uplo, diag):
    T = np.tril(Am, -1) if uplo == "lower" else np.triu(Am, 1)
    return T + (np.eye(len(Am)) if diag == "unit" else np.diag(np.diag(Am)))


@pytest.mark.parametrize("layout", LAYOUTS)
@pytest.mark.parametrize("side", ["left", "right"])
@pytest.mark.parametrize("uplo", ["lower", "upper"])
@pytest.mark.parametrize("routine", ["ssymm", "dsymm"])
def test_symm(env, layout, side, uplo, routine):
    wg, dev, _ = env
    dt = np.float64 if routine == "dsymm" else np.float32
    rng = np.random.default_rng(4)
    m, n = 5, 7
    order = m if side == "left" else n
    A, lda = stored(order, order, layout, 1, rng, dt)
    B, ldb = stored(m, n, layout, 2, rng, dt)
    C, ldc = stored(m, n, layout, 1, rng, dt)
    got = getattr(wg, routine)(dev, side, uplo, m, n, 1.25, A, lda, B, ldb, -1.0, C, ldc, layout)["C"]
    Am = mat(A, lda, order, order, layout)[0]
    L = np.tril(Am) if uplo == "lower" else np.triu(Am)
    S = L + L.T - np.diag(np.diag(Am))
    Bm = mat(B, ldb, m, n, layout)[0]
    Cm, idx = mat(C, ldc, m, n, layout)
    want = 1.25 * (S @ Bm if side == "left" else Bm @ S) - Cm
    check_block(got, C, idx, want)


@pytest.mark.parametrize("layout", LAYOUTS)
@pytest.mark.parametrize("side", ["left", "right"])
@pytest.mark.parametrize("uplo", ["lower", "upper"])
@pytest.mark.parametrize("tA", TRANS)
@pytest.mark.parametrize("routine", ["strmm", "dtrmm", "strsm"])
def test_triangular(env, layout, side, uplo, tA, routine):
    wg, dev, _ = env
    dt = np.float64 if routine == "dtrmm" else np.float32
    rng = np.random.default_rng(5)
    m, n = 6, 4
    order = m if side == "left" else n
    A, lda = stored(order, order, layout, 2, rng, dt)
    A[:] = A / order
    Am = mat(A, lda, order, order, layout)[0]
    diag = "unit" if tA == "transpose" else "non-unit"
    if diag == "non-unit":
        d = mat(A, lda, order, order, layout)[1][np.arange(order), np.arange(order)]
        A[d] = 2.0
        Am = mat(A, lda, order, order, layout)[0]
    B, ldb = stored(m, n, layout, 1, rng, dt)
    Bm, idx = mat(B, ldb, m, n, layout)
    T = op(tri_of(Am, uplo, diag), tA)
    got = getattr(wg, routine)(dev, side, uplo, tA, diag, m, n, 1.5, A, lda, B, ldb, layout)["B"]
    if routine.endswith("trmm"):
        want = 1.5 * (T @ Bm if side == "left" else Bm @ T)
    else:
        want = np.linalg.solve(T, 1.5 * Bm) if side == "left" else np.linalg.solve(T.T, 1.5 * Bm.T).T
    check_block(got, B, idx, want)


@pytest.mark.parametrize("la,lb", [("row-major", "column-major"), ("column-major", "row-major")])
@pytest.mark.parametrize("routine", ["strsm", "strmm"])
def test_triangular_gpu_matrices_with_mixed_layouts(env, la, lb, routine):
    wg, dev, _ = env
    rng = np.random.default_rng(6)
    m, n = 3, 5
    A, lda = stored(n, n, la, 0, rng)
    d = mat(A, lda, n, n, la)[1][np.arange(n), np.arange(n)]
    A[d] = 3.0
    B, ldb = stored(m, n, lb, 0, rng)
    GA = wg.GpuMatrix.from_(dev, A, n, n, lda, la)
    GB = wg.GpuMatrix.from_(dev, B, m, n, ldb, lb)
    assert getattr(wg, routine)(dev, "right", "upper", "transpose", "non-unit", m, n, 0.5, GA, lda, GB, ldb) == {}
    got = GB.read()
    T = tri_of(mat(A, lda, n, n, la)[0], "upper", "non-unit").T
    Bm = mat(B, ldb, m, n, lb)[0]
    want = 0.5 * Bm @ T if routine == "strmm" else np.linalg.solve(T.T, 0.5 * Bm.T).T
    assert np.allclose(got.reshape((m, n) if lb == "row-major" else (n, m)),
                       want if lb == "row-major" else want.T, rtol=2e-5, atol=2e-5)


@pytest.mark.parametrize("layout", LAYOUTS)
@pytest.mark.parametrize("trans", TRANS)
@pytest.mark.parametrize("routine", ["sgemv", "dgemv"])
@pytest.mark.parametrize("gpu", [False, True])
def test_gemv(env, layout, trans, routine, gpu):
    wg, dev, fake = env
    dt = np.float64 if routine == "dgemv" else np.float32
    rng = np.random.default_rng(7)
    m, n, incx, incy = 6, 4, 2, 3
    A, lda = stored(m, n, layout, 1, rng, dt)
    xlen, ylen = (n, m) if trans == "no-transpose" else (m, n)
    x = (rng.random((xlen - 1) * incx + 1) * 2 - 1).astype(dt)
    y = (rng.random((ylen - 1) * incy + 1) * 2 - 1).astype(dt)
    fn = getattr(wg, routine)
    if gpu:
        GA = wg.GpuMatrix.from_(dev, A, m, n, lda, layout)
        gx, gy = wg.GpuVector.from_(dev, x), wg.GpuVector.from_(dev, y)
        assert fn(dev, trans, m, n, 0.5, GA, lda, gx, incx, 1.5, gy, incy) == {}
        got = gy.read()
    else:
        got = fn(dev, trans, m, n, 0.5, A, lda, x, incx, 1.5, y, incy, layout)["y"]
    Am = mat(A, lda, m, n, layout)[0]
    want = 0.5 * op(Am, trans) @ x[np.arange(xlen) * incx] + 1.5 * y[np.arange(ylen) * incy]
    iy = np.arange(ylen) * incy
    check_block(got, y, iy, want)
    # the column-major frame: row-major A flips the transpose
    kind, _, t_cm, m_cm, n_cm = fake.calls[-1]
    assert (t_cm == 1) == ((trans == "no-transpose") == (layout == "row-major"))
    assert (m_cm, n_cm) == ((m, n) if layout == "column-major" else (n, m))


def test_quick_returns_and_zero_dimensions(env):
    wg, dev, fake = env
    y = np.arange(5, dtype=np.float64)
    r = wg.dgemv(dev, "no-transpose", 5, 5, 0.0, np.ones(25), 5, np.ones(5), 1, 1.0, y, 1)
    assert r["y"] is y and not fake.calls
    B = np.arange(8, dtype=np.float32)
    assert wg.strsm(dev, "left", "lower", "no-transpose", "non-unit", 0, 4, 1.0, np.zeros(0, np.float32), 1, B,
                    4)["B"] is B
    C = np.arange(6, dtype=np.float64)
    assert wg.dgemm(dev, "no-transpose", "no-transpose", 2, 3, 0, 0.5, np.zeros(8), 2, np.zeros(8), 3, 1.0, C,
                    3)["C"] is C
    assert not fake.calls
