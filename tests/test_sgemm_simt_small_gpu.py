"""The small-tile FFMA kernel (32 x 64 tiles of C, a cp.async ring of 16-deep
k-tiles): bit for bit the oracle's FMA restatement at tile edges, depths that
end inside a k-tile (no padded term is added), every transpose, gemmtr
triangles, and beta = 0 ignoring C's NaNs. Leading dimensions that are
multiples of 4 ("vec") take the 16-byte copies, with partial zero-filled copies
at the edges; the others ("tight", "odd") the 4-byte ones."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import bits_equal

pytestmark = pytest.mark.gpu
T, N = "transpose", "no-transpose"
TR = {N: 0, T: 1}


@pytest.fixture
def small(device):
    device.set_sgemm_path("simt_small")
    yield device
    device.set_sgemm_path("auto")


def _ld(rows, pad):
    return {"tight": rows, "odd": rows + 3, "vec": (rows + 3) // 4 * 4 + 4}[pad]


def _case(wg, ta, tb, m, n, k, pad, seed):
    aR, aC = (m, k) if ta == N else (k, m)
    bR, bC = (k, n) if tb == N else (n, k)
    lda, ldb, ldc = _ld(aR, pad), _ld(bR, pad), _ld(m, pad)
    A = wg.randomFloat32Array(lda * aC, -1, 1, seed)
    B = wg.randomFloat32Array(ldb * bC, -1, 1, seed + 1)
    C = wg.randomFloat32Array(ldc * n, -1, 1, seed + 2)
    return A, lda, B, ldb, C, ldc


@pytest.mark.parametrize("shape", [(1, 1, 1), (1, 70, 15), (33, 1, 16), (31, 63, 17), (32, 64, 32),
                                   (65, 129, 95), (200, 130, 1), (96, 192, 160)])
@pytest.mark.parametrize("ta,tb", [(N, N), (T, N), (N, T), (T, T)])
@pytest.mark.parametrize("pad", ["tight", "odd", "vec"])
def test_tile_edges_bit_exact(wg, device, oracle, small, shape, ta, tb, pad):
    m, n, k = shape
    A, lda, B, ldb, C, ldc = _case(wg, ta, tb, m, n, k, pad, 7 + m + n + k + len(pad))
    device.profile_read()
    device.set_profiling(True)
    try:
        got = wg.sgemm(device, ta, tb, m, n, k, 1.25, A, lda, B, ldb, -0.5, C, ldc, "column-major")["C"]
    finally:
        device.set_profiling(False)
    assert device.profile_read().get("sgemm_simt_small", (0,))[0] >= 1
    want = oracle.sgemm(TR[ta], TR[tb], m, n, k, 1.25, A, lda, B, ldb, -0.5, C, ldc, variant=1)
    assert bits_equal(got, want)


def test_beta_zero_ignores_c(wg, device, oracle, small):
    m, n, k = 100, 90, 40
    A, lda, B, ldb, C, ldc = _case(wg, N, N, m, n, k, "vec", 91)
    C[::7] = np.nan
    got = wg.sgemm(device, N, N, m, n, k, 0.75, A, lda, B, ldb, 0.0, C, ldc, "column-major")["C"]
    want = oracle.sgemm(0, 0, m, n, k, 0.75, A, lda, B, ldb, 0.0, C, ldc, variant=1)
    assert bits_equal(got, want)
    assert not np.any(np.isnan(got.reshape(n, ldc)[:, :m]))


@pytest.mark.parametrize("uplo", ["lower", "upper"])
def test_gemmtr_triangle(wg, device, oracle, small, uplo):
    from test_gemmtr_gpu import call, check_against, random_case

    case = random_case("sgemmtr", uplo, "column-major", n=150, k=45, m=170, seed=23)
    got = call(wg, device, case, case["A"], case["B"], case["C"])["C"]
    check_against(oracle, case, got, exact=True)
