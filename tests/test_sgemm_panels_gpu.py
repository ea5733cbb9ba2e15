"""Panelled 3xTF32 products on the GPU. They back the typed-array sgemm above
2 GFLOP and the sharded sgemm. Two forms: with the fused kernel (each panel one
launch that splits its own operands) a value outside the split's range sends
only the 128 x BN tiles it touches to the FFMA kernel; with the split pass
(op(A) split once, each op(B) panel split on a side stream while the previous
panel's MMA runs; forced by 'tf32x3_packed', and taken for operands the fused
kernel's tensor maps cannot describe) one bad op(B) value sends its panel, one
bad op(A) value sends every panel. Both are checked against the oracle."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import bits_equal
from gemm_check import check_sgemm

pytestmark = pytest.mark.gpu
N = "no-transpose"


def host_panels(m, n, k):
    """Panel width of the typed-array path (its rule, restated)."""
    if 2.0 * m * n * k < 2e9 or n < 512:
        return n
    p = -(-n // 4)
    p = -(-p // 256) * 256
    return min(p, n)


@pytest.fixture
def packed(device):
    device.set_sgemm_path("tf32x3_packed")
    yield device
    device.set_sgemm_path("auto")


@pytest.fixture
def fused256(device):
    device.set_sgemm_path("tf32x3_fused_bn256")
    yield device
    device.set_sgemm_path("auto")


def _inputs(wg, m, n, k, seed):
    A = wg.randomFloat32Array(m * k, -1, 1, seed)
    B = wg.randomFloat32Array(k * n, -1, 1, seed + 1)
    C = wg.randomFloat32Array(m * n, -1, 1, seed + 2)
    return A, B, C


@pytest.mark.parametrize("shape", [(1024, 1040, 1100), (1100, 2048, 900)])
def test_host_array_panels_match_oracle(wg, device, oracle, shape):
    m, n, k = shape
    panel = host_panels(m, n, k)
    panels = -(-n // panel)
    assert panels > 1
    A, B, C = _inputs(wg, m, n, k, 40)
    before = device.sgemm_stats()
    got = wg.sgemm(device, N, N, m, n, k, 0.75, A, m, B, k, -0.5, C, m, "column-major")["C"]
    after = device.sgemm_stats()
    assert after["tf32x3_launches"] - before["tf32x3_launches"] == panels
    assert after["fallbacks"] == before["fallbacks"]
    check_sgemm(oracle, got, N, N, m, n, k, 0.75, A, m, B, k, -0.5, C, m, "column-major")


def test_bad_b_panel_falls_back_alone(wg, device, oracle, packed):
    m, n, k = 1024, 2048, 1024
    panel = host_panels(m, n, k)
    A, B, C = _inputs(wg, m, n, k, 50)
    j_bad = panel + 17  # a column of op(B) in the second panel
    B[3 + j_bad * k] = np.inf
    before = device.sgemm_stats()
    got = wg.sgemm(device, N, N, m, n, k, 1.0, A, m, B, k, 1.0, C, m, "column-major")["C"]
    assert device.sgemm_stats()["fallbacks"] == before["fallbacks"] + 1
    want = oracle.sgemm(0, 0, m, n, k, 1.0, A, m, B, k, 1.0, C, m, variant=1)
    # the flagged panel ran on the FFMA kernel: bit for bit the FMA restatement
    lo, hi = panel * m, 2 * panel * m
    assert bits_equal(got[lo:hi], want[lo:hi])
    # the others stayed on the tensor cores, within the bound
    for j0, j1 in ((0, panel), (2 * panel, n)):
        sub = slice(j0 * m, j1 * m)
        check_sgemm(oracle, got[sub], N, N, m, j1 - j0, k, 1.0, A, m, B[j0 * k:], k, 1.0, C[sub], m,
                    "column-major")


def test_bad_a_sends_every_panel_back(wg, device, oracle, packed):
    m, n, k = 1024, 1536, 1024
    panels = -(-n // host_panels(m, n, k))
    A, B, C = _inputs(wg, m, n, k, 60)
    A[7 + 100 * m] = np.nan
    before = device.sgemm_stats()
    got = wg.sgemm(device, N, N, m, n, k, 1.25, A, m, B, k, 0.0, C, m, "column-major")["C"]
    assert device.sgemm_stats()["fallbacks"] == before["fallbacks"] + panels
    want = oracle.sgemm(0, 0, m, n, k, 1.25, A, m, B, k, 0.0, C, m, variant=1)
    assert bits_equal(got, want)


def test_clean_call_after_flagged_panels(wg, device, oracle, packed):
    """Flags of one product do not leak into the next."""
    test_bad_b_panel_falls_back_alone(wg, device, oracle, packed)
    m, n, k = 1024, 1040, 1100
    A, B, C = _inputs(wg, m, n, k, 70)
    before = device.sgemm_stats()
    got = wg.sgemm(device, N, N, m, n, k, 1.0, A, m, B, k, 0.5, C, m, "column-major")["C"]
    assert device.sgemm_stats()["fallbacks"] == before["fallbacks"]
    check_sgemm(oracle, got, N, N, m, n, k, 1.0, A, m, B, k, 0.5, C, m, "column-major")


@pytest.mark.parametrize("kind", ["tf32x3_packed", "tf32x3_fused_bn256"])
def test_sharded_single_rank_panels_with_bad_panel(wg, device, oracle, kind):
    """The sharded sgemm on one rank with explicit 256-column panels: the same
    product path. With either kernel the bad value's 256 columns (its panel, or
    its 128 x 256 tiles in every row block) fall back."""
    device.set_sgemm_path(kind)
    from wgblas_b200.shard import Comm, gemm_sharded

    m, n, k = 640, 1280, 512
    A, B, C = _inputs(wg, m, n, k, 80)
    B[5 + 700 * k] = -np.inf  # column 700: the third 256-column panel
    GA = wg.GpuMatrix.from_(device, A, m, k, m, "column-major")
    GB = wg.GpuMatrix.from_(device, B, k, n, k, "column-major")
    GC = wg.GpuMatrix.from_(device, C, m, n, m, "column-major")
    comm = Comm(device, 1, 0, Comm.unique_id(), timeout_ms=30000)
    try:
        before = device.sgemm_stats()
        gemm_sharded(comm, False, False, m, n, k, 1.0, GA, GB, -1.0, GC, root=0, panel_cols=256)
        comm.wait()
        got = GC.read()
        after = device.sgemm_stats()
    finally:
        device.set_sgemm_path("auto")
        comm.destroy()
        for g in (GA, GB, GC):
            g.destroy()
    assert after["tf32x3_launches"] - before["tf32x3_launches"] == 5
    assert after["fallbacks"] == before["fallbacks"] + 1
    want = oracle.sgemm(0, 0, m, n, k, 1.0, A, m, B, k, -1.0, C, m, variant=1)
    assert bits_equal(got[512 * m:768 * m], want[512 * m:768 * m])
    for j0, j1 in ((0, 512), (768, n)):
        sub = slice(j0 * m, j1 * m)
        check_sgemm(oracle, got[sub], N, N, m, j1 - j0, k, 1.0, A, m, B[j0 * k:], k, -1.0, C[sub], m,
                    "column-major")


def test_fused_bad_b_tiles_fall_back_alone(wg, device, oracle, fused256):
    """Fused panels: one Inf in op(B) sends the 128 x 256 tiles of its column block
    (every row block of one panel's tile column) to the FFMA kernel, bit for bit
    the FMA restatement there; every other column stays on the tensor cores."""
    m, n, k = 1024, 2048, 1024
    panel = host_panels(m, n, k)
    A, B, C = _inputs(wg, m, n, k, 50)
    j_bad = panel + 17
    B[3 + j_bad * k] = np.inf
    t0 = (j_bad - panel) // 256 * 256 + panel  # first column of its tile
    before = device.sgemm_stats()
    got = wg.sgemm(device, N, N, m, n, k, 1.0, A, m, B, k, 1.0, C, m, "column-major")["C"]
    assert device.sgemm_stats()["fallbacks"] == before["fallbacks"] + 1
    want = oracle.sgemm(0, 0, m, n, k, 1.0, A, m, B, k, 1.0, C, m, variant=1)
    assert bits_equal(got[t0 * m:(t0 + 256) * m], want[t0 * m:(t0 + 256) * m])
    for j0, j1 in ((0, t0), (t0 + 256, n)):
        sub = slice(j0 * m, j1 * m)
        check_sgemm(oracle, got[sub], N, N, m, j1 - j0, k, 1.0, A, m, B[j0 * k:], k, 1.0, C[sub], m,
                    "column-major")


def test_fused_bad_a_row_block_in_every_panel(wg, device, oracle, fused256):
    """Fused panels: one NaN in op(A) row 7 sends tile row 0 of every panel to the
    FFMA kernel; the other row blocks stay on the tensor cores."""
    m, n, k = 1024, 1536, 1024
    panels = -(-n // host_panels(m, n, k))
    A, B, C = _inputs(wg, m, n, k, 60)
    A[7 + 100 * m] = np.nan
    before = device.sgemm_stats()
    got = wg.sgemm(device, N, N, m, n, k, 1.25, A, m, B, k, 0.0, C, m, "column-major")["C"]
    assert device.sgemm_stats()["fallbacks"] == before["fallbacks"] + panels
    want = oracle.sgemm(0, 0, m, n, k, 1.25, A, m, B, k, 0.0, C, m, variant=1)
    G, W = got.reshape(n, m), want.reshape(n, m)
    assert bits_equal(np.ascontiguousarray(G[:, :128]), np.ascontiguousarray(W[:, :128]))
    A2 = A.copy()
    A2[7 + 100 * m] = 0.0
    truth, absab = oracle.sgemm_truth(0, 0, m, n, k, 1.25, A2, m, B, k, 0.0, C, m)
    bound = oracle.sgemm_bound(m, n, k, 1.25, absab, 0.0, C, m)[128:]
    err = np.abs(oracle.block(got, m, n, m).astype(np.float64) - oracle.dense(truth, m, n))[128:]
    assert np.all(err <= bound)
