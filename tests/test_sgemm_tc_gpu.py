"""The 3xTF32 tensor-core sgemm (tcgen05/TMEM/TMA) against the oracle, forced on
through the dispatcher: ragged and aligned shapes, every transpose pair, the
device-side fallback to the FFMA kernel, and worst-case same-sign data."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import bits_equal
from gemm_check import check_sgemm, ieee_match

pytestmark = pytest.mark.gpu
T, N = "transpose", "no-transpose"


@pytest.fixture
def tc(device):
    device.set_sgemm_path("tf32x3")
    yield device
    device.set_sgemm_path("auto")


@pytest.fixture
def packed(device):
    """The split pass + MMA kernel, whose fallback covers the whole call (the fused
    kernel's per-tile fallback is tested in test_sgemm_fused_gpu.py)."""
    device.set_sgemm_path("tf32x3_packed")
    yield device
    device.set_sgemm_path("auto")


def _run(wg, dev, ta, tb, m, n, k, alpha, beta, layout="column-major", seed=7, low=-1.0, high=1.0, pad=(0, 0, 0)):
    cm = layout == "column-major"
    aR, aC = (m, k) if ta == N else (k, m)
    bR, bC = (k, n) if tb == N else (n, k)
    lda = (aR if cm else aC) + pad[0]
    ldb = (bR if cm else bC) + pad[1]
    ldc = (m if cm else n) + pad[2]
    A = wg.randomFloat32Array(lda * (aC if cm else aR), low, high, seed)
    B = wg.randomFloat32Array(ldb * (bC if cm else bR), low, high, seed + 1)
    C = wg.randomFloat32Array(ldc * (n if cm else m), low, high, seed + 2)
    got = wg.sgemm(dev, ta, tb, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, layout)["C"]
    return got, (ta, tb, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, layout)


@pytest.mark.parametrize("shape", [(128, 256, 64), (200, 300, 77), (512, 512, 512), (1000, 1023, 777),
                                   (129, 257, 40), (64, 640, 1000)])
@pytest.mark.parametrize("ta", [N, T])
@pytest.mark.parametrize("tb", [N, T])
def test_tc_shapes_and_transposes(wg, device, oracle, tc, shape, ta, tb):
    m, n, k = shape
    before = device.sgemm_stats()
    got, args = _run(wg, device, ta, tb, m, n, k, 1.5, 0.5, pad=(3, 1, 2))
    after = device.sgemm_stats()
    assert after["tf32x3_launches"] == before["tf32x3_launches"] + 1
    assert after["fallbacks"] == before["fallbacks"], "unexpected fallback to the FFMA kernel"
    rep = check_sgemm(oracle, got, *args)
    assert rep["forward_factor"] <= 1


@pytest.mark.parametrize("layout", ["row-major", "column-major"])
@pytest.mark.parametrize("beta", [0.0, -2.0])
def test_tc_layouts_and_beta(wg, device, oracle, tc, layout, beta):
    got, args = _run(wg, device, T, N, 300, 260, 130, 0.3, beta, layout=layout, pad=(4, 0, 1))
    check_sgemm(oracle, got, *args)


def test_tc_same_sign_worst_case(wg, device, oracle, tc):
    """U[0,1] operands: every product has the same sign, so accumulation errors add
    up instead of cancelling — the hardest case for the tensor-core accumulator."""
    got, args = _run(wg, device, N, N, 256, 256, 4096, 1.0, 1.0, low=0.0, high=1.0, seed=90)
    rep = check_sgemm(oracle, got, *args)
    print("same-sign K=4096 worst bound fraction:", rep["max_bound_frac"])


@pytest.mark.parametrize("bad", [np.inf, -np.inf, np.nan, 1e-20, 3e20])
def test_tc_device_fallback(wg, device, oracle, packed, bad):
    """Operands the split cannot carry exactly make the pack pass flag the call on the
    device; the tensor-core kernel then exits and the FFMA kernel computes C."""
    m = n = k = 256
    A = wg.randomFloat32Array(m * k, -1, 1, 31)
    B = wg.randomFloat32Array(k * n, -1, 1, 32)
    C = wg.randomFloat32Array(m * n, -1, 1, 33)
    A[5 + 17 * m] = bad
    before = device.sgemm_stats()
    got = wg.sgemm(device, N, N, m, n, k, 1.25, A, m, B, k, 0.5, C, m, "column-major")["C"]
    assert device.sgemm_stats()["fallbacks"] == before["fallbacks"] + 1
    want = oracle.sgemm(0, 0, m, n, k, 1.25, A, m, B, k, 0.5, C, m, variant=1)
    assert bits_equal(got, want), "fallback result differs from the FMA restatement"
    if np.isfinite(bad):
        ieee_match(got, want, 0)


def test_tc_no_stale_fallback(wg, device, oracle, packed):
    """A flagged call does not send the next (clean) call to the fallback."""
    test_tc_device_fallback(wg, device, oracle, packed, np.inf)
    before = device.sgemm_stats()
    got, args = _run(wg, device, N, T, 256, 256, 256, 1.0, 0.0)
    assert device.sgemm_stats()["fallbacks"] == before["fallbacks"]
    check_sgemm(oracle, got, *args)


def test_tc_gpumatrix_and_workspace_growth(wg, device, oracle, tc):
    for (m, n, k) in [(256, 256, 64), (1024, 768, 512), (300, 200, 100)]:
        A = wg.randomFloat32Array(m * k, -1, 1, m)
        B = wg.randomFloat32Array(k * n, -1, 1, n)
        C = wg.randomFloat32Array(m * n, -1, 1, k)
        GA = wg.GpuMatrix.from_(device, A, m, k, m, "column-major")
        GB = wg.GpuMatrix.from_(device, B, k, n, k, "column-major")
        GC = wg.GpuMatrix.from_(device, C, m, n, m, "column-major")
        try:
            wg.sgemm(device, N, N, m, n, k, 2.0, GA, m, GB, k, -1.0, GC, m)
            got = GC.read()
        finally:
            for g in (GA, GB, GC):
                g.destroy()
        check_sgemm(oracle, got, N, N, m, n, k, 2.0, A, m, B, k, -1.0, C, m, "column-major")


def test_auto_picks_tc_for_large_k(wg, device, oracle):
    before = device.sgemm_stats()
    got, args = _run(wg, device, T, N, 1024, 1024, 1024, 1.0, 0.0)
    after = device.sgemm_stats()
    # host arrays this size arrive in column panels: one tensor-core launch per panel
    assert after["tf32x3_launches"] > before["tf32x3_launches"]
    assert after["simt_launches"] == before["simt_launches"]
    check_sgemm(oracle, got, *args)


def test_auto_picks_small_ffma_for_small_products(wg, device, oracle):
    """512^3 (128 tiles of 32 x 64, one per SM, 32 k-tiles deep): the small-tile
    FFMA kernel, bit for bit the FMA restatement."""
    before = device.sgemm_stats()
    device.profile_read()
    device.set_profiling(True)
    try:
        got, args = _run(wg, device, N, N, 512, 512, 512, 1.5, 0.5)
    finally:
        device.set_profiling(False)
    after = device.sgemm_stats()
    assert after["tf32x3_launches"] == before["tf32x3_launches"]
    assert after["simt_launches"] == before["simt_launches"] + 1
    assert device.profile_read().get("sgemm_simt_small", (0,))[0] == 1
    rep = check_sgemm(oracle, got, *args, exact=True)
    assert rep is not None
