"""strsm on the GPU, following the reference's tests/strsm/src/test.strsm.js:
its edge cases and validation specs, the single-block and many-block in-place
paths at every side / uplo / transA / layout (backward residual factor <= 5 of
tests/strsm/helpers.js, leading-dimension padding unchanged), the IEEE
special-value rules against the restated stdlib oracle, alpha = 0 and zero
dimensions, GpuMatrix operands in place, and solves large enough that the
updates between diagonal blocks run on the 3xTF32 tensor-core GEMM."""
from __future__ import annotations

import math

import numpy as np
import pytest

import validation_runner as vr
from conftest import bits_equal, load_golden

pytestmark = pytest.mark.gpu
THRESHOLD = 5.0  # tests/strsm/src/test.strsm.js:22


def run(wg, device, a, B=None):
    side, uplo, transA, diag, m, n, alpha, A, lda, B0, ldb, layout = a
    return wg.strsm(device, side, uplo, transA, diag, m, n, alpha, A, lda, B0 if B is None else B, ldb,
                    layout)["B"]


def padding_mask(m, n, ld, layout, size):
    i = np.arange(m)[:, None]
    j = np.arange(n)[None, :]
    idx = (j * ld + i) if layout == "column-major" else (i * ld + j)
    pad = np.ones(size, bool)
    pad[idx.ravel()] = False
    return pad


@pytest.fixture(params=["recursive", "flow"])
def strsm_path(request, device):
    """Runs a test on both solve forms: GEMM updates with a launch per block, and
    the cooperative flow kernel."""
    device.set_strsm_path(request.param)
    yield request.param
    device.set_strsm_path("auto")


def check(oracle, got, a, pad_check=True):
    factor = oracle.strsm_residual_factor(got, *a)
    assert factor <= THRESHOLD, factor
    if pad_check:
        side, uplo, transA, diag, m, n, alpha, A, lda, B, ldb, layout = a
        pad = padding_mask(m, n, ldb, layout, B.size)
        assert bits_equal(got[pad], B[pad]), "padding changed"


@pytest.mark.parametrize("case", load_golden("strsm_edge_cases.json"), ids=lambda c: c["label"][:50])
def test_edge_cases(wg, device, oracle, case):
    a = (case["side"], case["uplo"], case["transA"], case["diag"], case["m"], case["n"], case["alpha"],
         np.array(case["A"], np.float32), case["lda"], np.array(case["B"], np.float32), case["ldb"], case["layout"])
    got = run(wg, device, a)
    check(oracle, got, a)
    assert np.allclose(got, np.array(case["expected"], np.float32), rtol=2.0**-20, atol=0)
    assert bits_equal(a[9], np.array(case["B"], np.float32)), "the input B was modified"


def test_validation_specs(wg, device):
    for label, args, err in vr.cases("strsm", device, "invalid"):
        with pytest.raises(wg.Error) as ei:
            vr.call(wg.strsm, args)
        assert err in str(ei.value), label
    n = 0
    for label, args, _ in vr.cases("strsm", device, "edge"):
        assert "B" in vr.call(wg.strsm, args), label
        n += 1
    assert n >= 10


def test_alpha_zero_gives_literal_zeros(wg, device):
    B = np.array([math.inf, math.nan, 3, 4], np.float32)
    got = wg.strsm(device, "left", "lower", "no-transpose", "non-unit", 2, 2, 0.0, np.array([1, 0, 1, 1], np.float32),
                   2, B, 2)["B"]
    assert bits_equal(got, np.zeros(4, np.float32))


def test_zero_dimensions_leave_b(wg, device):
    for m, n, seed in ((0, 4, 300), (4, 0, 301)):
        B = wg.randomFloat32Array(16, -5, 5, seed)
        got = wg.strsm(device, "left", "lower", "no-transpose", "non-unit", m, n, 1.5, np.zeros(0, np.float32), 1,
                       B, 4)["B"]
        assert bits_equal(got, B)


def reference_system(wg, N, other, pad, side, layout, seed_a, seed_b):
    """The systems of tests/strsm/src/test.strsm.js:265-331 and :333-405:
    off-diagonals in [-1/N, 1/N), diagonal 2, B in [-1, 1) with padded ldb."""
    m, n = (N, other) if side == "left" else (other, N)
    cm = layout == "column-major"
    ld = (m if cm else n) + pad
    A = wg.randomFloat32Array(N * N, -1 / N, 1 / N, seed_a)
    A[np.arange(N) * (N + 1)] = 2.0
    B = wg.randomFloat32Array((n if cm else m) * ld, -1, 1, seed_b)
    return m, n, A, B, ld


@pytest.mark.parametrize("N,other", [(64, 70), (37, 7), (1, 7)])
@pytest.mark.parametrize("layout", ["row-major", "column-major"])
@pytest.mark.parametrize("side", ["left", "right"])
@pytest.mark.parametrize("uplo", ["lower", "upper"])
@pytest.mark.parametrize("transA", ["no-transpose", "transpose"])
def test_single_block(wg, device, oracle, strsm_path, N, other, layout, side, uplo, transA):
    m, n, A, B, ld = reference_system(wg, N, other, 3, side, layout, 121, 122)
    diag = "unit" if uplo == "upper" else "non-unit"
    a = (side, uplo, transA, diag, m, n, 1.5, A, N, B, ld, layout)
    check(oracle, run(wg, device, a), a)


@pytest.mark.parametrize("N,other,pad", [(150, 70, 1), (600, 200, 4)])
@pytest.mark.parametrize("layout", ["row-major", "column-major"])
@pytest.mark.parametrize("side", ["left", "right"])
@pytest.mark.parametrize("uplo", ["lower", "upper"])
@pytest.mark.parametrize("transA", ["no-transpose", "transpose"])
def test_many_blocks_in_place(wg, device, oracle, strsm_path, N, other, pad, layout, side, uplo, transA):
    m, n, A, B, ld = reference_system(wg, N, other, pad, side, layout, 101, 102)
    diag = "unit" if transA == "transpose" else "non-unit"
    a = (side, uplo, transA, diag, m, n, 1.5, A, N, B, ld, layout)
    check(oracle, run(wg, device, a), a)


@pytest.mark.parametrize("side,uplo", [("left", "lower"), ("left", "upper"), ("right", "lower")])
def test_two_blocks(wg, device, oracle, strsm_path, side, uplo):
    order, other = 70, 5
    m, n = (order, other) if side == "left" else (other, order)
    rng = np.random.default_rng(7)
    A = (rng.random(order * order) - 0.5).astype(np.float32)
    A[np.arange(order) * (order + 1)] = (5 + 10 * rng.random(order)).astype(np.float32)
    B = wg.randomFloat32Array(m * n, -1, 1, 8)
    a = (side, uplo, "no-transpose", "non-unit", m, n, 1.0, A, order, B, n, "row-major")
    check(oracle, run(wg, device, a), a)


def assert_ieee_match(got, want, tol=1e-4):
    """tests/helpers/specials.js assertIeeeMatch: NaN <-> NaN, the same signed
    Infinity, finite values within tol relative (absolute near zero)."""
    g = got.astype(np.float64)
    w = want.astype(np.float64)
    nan = np.isnan(w)
    assert np.all(np.isnan(g[nan]))
    inf = np.isinf(w)
    assert np.all(g[inf] == w[inf])
    fin = ~nan & ~inf
    assert np.all(np.isfinite(g[fin]))
    assert np.all(np.abs(g[fin] - w[fin]) <= tol * np.maximum(1.0, np.abs(w[fin])))


@pytest.mark.parametrize("uplo", ["lower", "upper"])
@pytest.mark.parametrize("transA", ["no-transpose", "transpose"])
@pytest.mark.parametrize("m", [7, 600])
@pytest.mark.parametrize("label", ["inf early in B", "inf mid B", "-inf late in B", "inf in A"])
def test_ieee_special_values(wg, device, oracle, strsm_path, uplo, transA, m, label):
    """tests/strsm/src/test.strsm.js:498-578: Infinity in B or in A's referenced
    triangle lands where substitution puts it; NaN in the other triangle is never read."""
    n = 5

    def at(cols, r, c):
        return r * cols + c

    A = wg.randomFloat32Array(m * m, -1, 1, 1)
    A[np.arange(m) * (m + 1)] += m + 4
    A[at(m, 1, 4) if uplo == "lower" else at(m, 4, 1)] = np.nan
    B = wg.randomFloat32Array(m * n, -1, 1, 2)
    if label == "inf early in B":
        B[at(n, 1, 2)] = np.inf
    elif label == "inf mid B":
        B[at(n, m // 2, 0)] = np.inf
    elif label == "-inf late in B":
        B[at(n, m - 2, 4)] = -np.inf
    else:
        A[at(m, m - 1, 2) if uplo == "lower" else at(m, 2, m - 1)] = np.inf
    a = ("left", uplo, transA, "non-unit", m, n, 1.0, A, m, B, n, "row-major")
    assert_ieee_match(run(wg, device, a), oracle.strsm(*a))


@pytest.mark.parametrize("a_layout,b_layout", [("column-major", "column-major"), ("row-major", "column-major"),
                                               ("column-major", "row-major")])
def test_gpumatrix_in_place(wg, device, oracle, strsm_path, a_layout, b_layout):
    """GpuMatrix operands are solved in place; A and B may carry different layouts."""
    order, other = 300, 130
    rng = np.random.default_rng(11)
    A = ((rng.random(order * order) * 2 - 1) / order).astype(np.float32)
    A[np.arange(order) * (order + 1)] = 2.0
    m, n = other, order  # side right
    ldb = m if b_layout == "column-major" else n
    B = (rng.random(m * n) * 2 - 1).astype(np.float32)
    GA = wg.GpuMatrix.from_(device, A, order, order, order, a_layout)
    GB = wg.GpuMatrix.from_(device, B, m, n, ldb, b_layout)
    try:
        r = wg.strsm(device, "right", "upper", "transpose", "non-unit", m, n, 0.75, GA, order, GB, ldb)
        assert "B" not in r
        got = GB.read()
    finally:
        GA.destroy()
        GB.destroy()
    if a_layout != b_layout:
        # The check restates a single layout: re-store A in B's layout.
        A = A.reshape(order, order).T.copy().ravel()
    check(oracle, got, ("right", "upper", "transpose", "non-unit", m, n, 0.75, A, order, B, ldb, b_layout),
          pad_check=False)


@pytest.mark.parametrize("side,uplo,transA", [("left", "lower", "no-transpose"), ("right", "upper", "transpose"),
                                              ("left", "upper", "transpose")])
def test_tensor_core_updates(wg, device, oracle, side, uplo, transA):
    """Orders 1000+ put the updates between diagonal blocks of the recursive form
    on the 3xTF32 GEMM."""
    order, other = (1024, 512) if side == "left" else (777, 900)
    m, n = (order, other) if side == "left" else (other, order)
    rng = np.random.default_rng(12)
    A = ((rng.random(order * order) * 2 - 1) / order).astype(np.float32)
    A[np.arange(order) * (order + 1)] = (1.5 + rng.random(order)).astype(np.float32)
    B = (rng.random(m * n) * 2 - 1).astype(np.float32)
    before = device.sgemm_stats()["tf32x3_launches"]
    a = (side, uplo, transA, "non-unit", m, n, -0.5, A, order, B, m, "column-major")
    device.set_strsm_path("recursive")
    device.set_sgemm_path("tf32x3")  # auto sends updates this small to the FFMA kernel
    try:
        got = run(wg, device, a)
    finally:
        device.set_strsm_path("auto")
        device.set_sgemm_path("auto")
    assert device.sgemm_stats()["tf32x3_launches"] > before
    check(oracle, got, a)


@pytest.mark.parametrize("side,uplo,transA,order,other", [
    ("left", "lower", "no-transpose", 200, 70),      # ragged last block and chunk
    ("right", "lower", "transpose", 1000, 513),      # one launch, several chunks
    ("left", "upper", "no-transpose", 130, 10000),   # more chunks than fit at once: several launches
    ("right", "upper", "no-transpose", 4096, 64),    # the bench's shape, one chunk of 64 blocks
])
def test_flow_shapes(wg, device, oracle, side, uplo, transA, order, other):
    """The flow form at shapes that exercise its partition: ragged blocks and
    right-hand-side chunks, several CTAs per chunk, and more chunks than one
    cooperative launch holds."""
    m, n = (order, other) if side == "left" else (other, order)
    rng = np.random.default_rng(order + other)
    A = ((rng.random(order * order) * 2 - 1) / order).astype(np.float32)
    A[np.arange(order) * (order + 1)] = (1.5 + rng.random(order)).astype(np.float32)
    B = (rng.random(m * n) * 2 - 1).astype(np.float32)
    a = (side, uplo, transA, "non-unit", m, n, 0.75, A, order, B, m, "column-major")
    device.set_strsm_path("flow")
    try:
        got = run(wg, device, a)
    finally:
        device.set_strsm_path("auto")
    check(oracle, got, a)
