"""The fused 3xTF32 sgemm (operands split inside the tcgen05 kernel, read by TMA
from the caller's matrices) against the oracle: every transpose pair and tile
width, ragged and aligned shapes, split-K plans, gemmtr triangles, and the
per-tile fallback to the FFMA kernel for operands outside the split's exact
range (those tiles bit for bit as the FMA restatement, the others within the
bound, C outside flagged tiles written once)."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import bits_equal
from gemm_check import check_sgemm, ieee_match

pytestmark = pytest.mark.gpu
T, N = "transpose", "no-transpose"
WIDTHS = ["tf32x3_fused_bn256", "tf32x3_fused_bn128", "tf32x3_fused_bn64", "tf32x3_pair"]


@pytest.fixture
def path(device):
    def set_path(p):
        device.set_sgemm_path(p)
    yield set_path
    device.set_sgemm_path("auto")


def _operands(wg, ta, tb, m, n, k, seed, low=-1.0, high=1.0, pad=(0, 0, 0)):
    """Column-major operands with leading dimensions rounded up to multiples of 4
    (plus pad*4), as the fused kernel's tensor maps need."""
    aR, aC = (m, k) if ta == N else (k, m)
    bR, bC = (k, n) if tb == N else (n, k)
    up = lambda x, p: (x + 3) // 4 * 4 + 4 * p  # noqa: E731
    lda, ldb, ldc = up(aR, pad[0]), up(bR, pad[1]), m + pad[2]
    A = wg.randomFloat32Array(lda * aC, low, high, seed)
    B = wg.randomFloat32Array(ldb * bC, low, high, seed + 1)
    C = wg.randomFloat32Array(ldc * n, low, high, seed + 2)
    return A, lda, B, ldb, C, ldc


@pytest.mark.parametrize("width", WIDTHS)
@pytest.mark.parametrize("shape", [(128, 256, 64), (200, 300, 77), (1000, 1023, 777), (64, 640, 1000), (37, 45, 9)])
@pytest.mark.parametrize("ta", [N, T])
@pytest.mark.parametrize("tb", [N, T])
def test_fused_shapes_transposes_widths(wg, device, oracle, path, width, shape, ta, tb):
    m, n, k = shape
    A, lda, B, ldb, C, ldc = _operands(wg, ta, tb, m, n, k, 7, pad=(1, 0, 3))
    path(width)
    before = device.sgemm_stats()
    got = wg.sgemm(device, ta, tb, m, n, k, 1.5, A, lda, B, ldb, 0.5, C, ldc, "column-major")["C"]
    after = device.sgemm_stats()
    assert after["tf32x3_launches"] == before["tf32x3_launches"] + 1
    assert after["fallbacks"] == before["fallbacks"], "unexpected fallback to the FFMA kernel"
    rep = check_sgemm(oracle, got, ta, tb, m, n, k, 1.5, A, lda, B, ldb, 0.5, C, ldc, "column-major")
    assert rep["forward_factor"] <= 1


@pytest.mark.parametrize("shape", [(512, 512, 512), (2048, 1024, 2048), (4096, 4096, 256), (300, 4000, 3000)])
def test_fused_auto_width_and_split_k(wg, device, oracle, path, shape):
    """Shapes whose plans cut the last wave's tiles into k-segments (the finishing
    segment adds the others' partial sums) and pick different tile widths."""
    m, n, k = shape
    A, lda, B, ldb, C, ldc = _operands(wg, T, N, m, n, k, 17)
    path("tf32x3")
    got = wg.sgemm(device, T, N, m, n, k, -0.75, A, lda, B, ldb, 1.25, C, ldc, "column-major")["C"]
    if m * n * k <= 2 ** 30:
        check_sgemm(oracle, got, T, N, m, n, k, -0.75, A, lda, B, ldb, 1.25, C, ldc, "column-major")
    else:
        from gemm_check import sampled_columns_truth

        cols = np.unique(np.linspace(0, n - 1, 24).astype(int))
        truth, absab, Cs = sampled_columns_truth(oracle, False, 1, 0, m, n, k, -0.75, A, lda, B, ldb, 1.25, C, ldc,
                                                 cols)
        g = np.stack([got[j * ldc: j * ldc + m] for j in cols], axis=1).astype(np.float64)
        bound = oracle.sgemm_bound(m, len(cols), k, -0.75, absab, 1.25, Cs, m)
        assert np.all(np.abs(g - oracle.dense(truth, m, len(cols))) <= bound)


def test_fused_same_sign_worst_case(wg, device, oracle, path):
    """U[0,1] operands: accumulation errors add up instead of cancelling."""
    m, n, k = 256, 256, 4096
    A, lda, B, ldb, C, ldc = _operands(wg, N, N, m, n, k, 90, low=0.0, high=1.0)
    path("tf32x3")
    got = wg.sgemm(device, N, N, m, n, k, 1.0, A, lda, B, ldb, 1.0, C, ldc, "column-major")["C"]
    rep = check_sgemm(oracle, got, N, N, m, n, k, 1.0, A, lda, B, ldb, 1.0, C, ldc, "column-major")
    print("fused same-sign K=4096 worst bound fraction:", rep["max_bound_frac"])


@pytest.mark.parametrize("width", WIDTHS)
@pytest.mark.parametrize("bad", [np.inf, -np.inf, np.nan, 1e-20, 3e20])
def test_fused_per_tile_fallback(wg, device, oracle, path, width, bad):
    """One element of A outside the split's range: the tiles of its row block go to
    the FFMA kernel (bit for bit the FMA restatement there, IEEE specials
    included); every other tile stays on the tensor cores, within the bound."""
    m, n, k = 384, 320, 200
    A, lda, B, ldb, C, ldc = _operands(wg, N, N, m, n, k, 31)
    row = 200  # tile row 1 of 3
    A[row + 17 * lda] = bad
    path(width)
    before = device.sgemm_stats()
    got = wg.sgemm(device, N, N, m, n, k, 1.25, A, lda, B, ldb, 0.5, C, ldc, "column-major")["C"]
    assert device.sgemm_stats()["fallbacks"] == before["fallbacks"] + 1
    want = oracle.sgemm(0, 0, m, n, k, 1.25, A, lda, B, ldb, 0.5, C, ldc, variant=1)
    G = got.reshape(n, ldc)[:, :m]
    W = want.reshape(n, ldc)[:, :m]
    flagged = slice(128, 256)
    assert bits_equal(np.ascontiguousarray(G[:, flagged]), np.ascontiguousarray(W[:, flagged]))
    ieee_match(got, want, 1e-4)
    # the other row blocks: clean tiles on the tensor cores, held to the bound
    clean = np.r_[0:128, 256:m]
    A2 = A.copy()
    A2[row + 17 * lda] = 0.0
    truth, absab = oracle.sgemm_truth(0, 0, m, n, k, 1.25, A2, lda, B, ldb, 0.5, C, ldc)
    t = oracle.dense(truth, m, n)[clean]
    bound = oracle.sgemm_bound(m, n, k, 1.25, absab, 0.5, C, ldc)[clean]
    g = oracle.block(got, m, n, ldc).astype(np.float64)[clean]
    assert np.all(np.abs(g - t) <= bound)
    assert bits_equal(got[m:ldc], C[m:ldc]), "padding of C was written"


def test_fused_fallback_in_one_k_segment(wg, device, oracle, path):
    """A split-K plan where only one k-segment of a tile sees the bad value: the
    finishing segment learns it through the tile's word and leaves C to the FFMA
    kernel; the next clean call on the same workspace does not fall back."""
    m, n, k = 1024, 1024, 2048
    A, lda, B, ldb, C, ldc = _operands(wg, N, N, m, n, k, 41)
    A[3 + 1900 * lda] = np.inf  # k index 1900: the last segment of tile row 0
    path("tf32x3_fused_bn256")

    def call():  # one call on resident operands (the typed-array path would cut B into panels)
        GA = wg.GpuMatrix.from_(device, A, m, k, lda, "column-major")
        GB = wg.GpuMatrix.from_(device, B, k, n, ldb, "column-major")
        GC = wg.GpuMatrix.from_(device, C, m, n, ldc, "column-major")
        try:
            wg.sgemm(device, N, N, m, n, k, 1.0, GA, lda, GB, ldb, 0.0, GC, ldc, "column-major")
            return GC.read()
        finally:
            for g in (GA, GB, GC):
                g.destroy()

    before = device.sgemm_stats()
    got = call()
    assert device.sgemm_stats()["fallbacks"] == before["fallbacks"] + 1
    want = oracle.sgemm(0, 0, m, n, k, 1.0, A, lda, B, ldb, 0.0, C, ldc, variant=1)
    G = got.reshape(n, m)  # [column, row]
    W = np.ascontiguousarray(oracle.block(want, m, n, ldc).T)
    assert bits_equal(np.ascontiguousarray(G[:, :128]), np.ascontiguousarray(W[:, :128]))
    assert np.all(np.isinf(G[:, 3]))
    A[3 + 1900 * lda] = 0.5
    before = device.sgemm_stats()
    got = call()
    assert device.sgemm_stats()["fallbacks"] == before["fallbacks"]
    full = C.copy()
    for j in range(n):
        full[j * ldc: j * ldc + m] = got[j * m:(j + 1) * m]
    check_sgemm(oracle, full, N, N, m, n, k, 1.0, A, lda, B, ldb, 0.0, C, ldc, "column-major")


@pytest.mark.parametrize("uplo", ["lower", "upper"])
@pytest.mark.parametrize("width", WIDTHS)
def test_fused_gemmtr_triangle(wg, device, oracle, path, uplo, width):
    n, k = 600, 300
    A = wg.randomFloat32Array(n * k, -1, 1, 51)
    B = wg.randomFloat32Array(k * n, -1, 1, 52)
    C = wg.randomFloat32Array(n * n, -1, 1, 53)
    path(width)
    got = wg.sgemmtr(device, uplo, N, N, n, n, k, 1.0, A, n, B, k, 0.5, C, n, "column-major")["C"]
    want = oracle.sgemmtr(1 if uplo == "lower" else 2, 0, 0, n, n, k, 1.0, A, n, B, k, 0.5, C, n)
    i, j = np.meshgrid(np.arange(n), np.arange(n), indexing="ij")
    inside = (j <= i) if uplo == "lower" else (j >= i)
    G = got.reshape(n, n).T  # [row, col]
    W = want.reshape(n, n).T
    Cm = C.reshape(n, n).T
    assert bits_equal(np.ascontiguousarray(G[~inside]), np.ascontiguousarray(Cm[~inside]))
    truth, absab = oracle.sgemm_truth(0, 0, n, n, k, 1.0, A, n, B, k, 0.5, C, n)
    bound = oracle.sgemm_bound(n, n, k, 1.0, absab, 0.5, C, n)
    err = np.abs(oracle.block(got, n, n, n).astype(np.float64) - oracle.dense(truth, n, n))
    assert np.all(err[inside] <= bound[inside])
    assert np.all(np.abs(G[inside].astype(np.float64) - W[inside]) <= bound[inside] * 2)


def test_fused_unaligned_operands_use_the_split_pass(wg, device, oracle, path):
    """Resident A with lda = 259 (not a multiple of 4): the tensor maps cannot
    describe it, so the call runs the split pass + MMA kernel; forcing the fused
    kernel is refused. (Typed-array calls never get here: their device copies
    have leading dimensions rounded up to multiples of 4.)"""
    m, n, k = 256, 256, 128
    A = wg.randomFloat32Array(259 * k, -1, 1, 61)
    B = wg.randomFloat32Array(k * n, -1, 1, 62)
    C = wg.randomFloat32Array(m * n, -1, 1, 63)
    GA = wg.GpuMatrix.from_(device, A, 259, k, 259, "column-major")
    GB = wg.GpuMatrix.from_(device, B, k, n, k, "column-major")
    GC = wg.GpuMatrix.from_(device, C, m, n, m, "column-major")
    try:
        path("tf32x3")
        device.profile_read()
        device.set_profiling(True)
        wg.sgemm(device, N, N, m, n, k, 1.0, GA, 259, GB, k, 0.0, GC, m, "column-major")
        device.set_profiling(False)
        assert "sgemm_tf32x3_pack" in device.profile_read()
        check_sgemm(oracle, GC.read(), N, N, m, n, k, 1.0, A, 259, B, k, 0.0, C, m, "column-major")
        path("tf32x3_fused_bn128")
        with pytest.raises(wg._native.NativeError):
            wg.sgemm(device, N, N, m, n, k, 1.0, GA, 259, GB, k, 0.0, GC, m, "column-major")
    finally:
        device.set_profiling(False)
        for g in (GA, GB, GC):
            g.destroy()
