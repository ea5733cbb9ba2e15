"""sgemv / dgemv on the GPU, following the reference's tests/sgemv/src/test.sgemv.js
and tests/dgemv/src/test.dgemv.js: the edge cases bit for bit, the validation
specs, seeded random fixtures and the split-chunk and long-row paths within
the reference's forward factor (tests/{sgemv,dgemv}/helpers.js), zero
dimensions, alpha = 0 and zero x entries with Infinity and NaN around, the
dgemv IEEE and exactness rules, GpuMatrix / GpuVector operands in place, and a
4096 x 4096 product per kernel."""
from __future__ import annotations

import math

import numpy as np
import pytest

import validation_runner as vr
from conftest import bits_equal, load_golden

pytestmark = pytest.mark.gpu
THRESHOLD = {"sgemv": 4.0, "dgemv": 5.0}  # test.sgemv.js:19, test.dgemv.js:33


def dtype_of(routine):
    return np.float64 if routine == "dgemv" else np.float32


def call(wg, device, routine, a):
    trans, m, n, alpha, A, lda, x, incx, beta, y, incy, layout = a
    return getattr(wg, routine)(device, trans, m, n, alpha, A, lda, x, incx, beta, y, incy, layout)


@pytest.mark.parametrize("case", load_golden("gemv_edge_cases.json"), ids=lambda c: f"{c['routine']}:{c['label'][:40]}")
def test_edge_cases_exact(wg, device, case):
    dt = dtype_of(case["routine"])
    a = (case["trans"], case["m"], case["n"], case["alpha"], np.array(case["A"], dt), case["lda"],
         np.array(case["x"], dt), case["incx"], case["beta"], np.array(case["y"], dt), case["incy"], case["layout"])
    got = call(wg, device, case["routine"], a)["y"]
    assert bits_equal(got, np.array(case["expected"], dt)), (got, case["expected"])
    assert bits_equal(a[9], np.array(case["y"], dt)), "the input y was modified"


@pytest.mark.parametrize("routine", ["sgemv", "dgemv"])
def test_validation_specs(wg, device, routine):
    fn = getattr(wg, routine)
    for label, args, err in vr.cases(routine, device, "invalid"):
        with pytest.raises(wg.Error) as ei:
            vr.call(fn, args)
        assert err in str(ei.value), label
    n = 0
    for label, args, _ in vr.cases(routine, device, "edge"):
        assert "y" in vr.call(fn, args), label
        n += 1
    assert n >= 10


def random_case(dt, trans, layout, m, n, incx, incy, seed, alpha=1.5, beta=0.75, pad=0):
    rng = np.random.default_rng(seed)
    cm = layout == "column-major"
    lda = (m if cm else n) + pad
    A = (rng.random(max(lda * (n if cm else m), 1)) * 2 - 1).astype(dt)
    no_t = trans == "no-transpose"
    xlen, ylen = (n, m) if no_t else (m, n)
    x = (rng.random(max((xlen - 1) * incx + 1, 1)) * 2 - 1).astype(dt)
    y = (rng.random(max((ylen - 1) * incy + 1, 1)) * 2 - 1).astype(dt)
    return (trans, m, n, alpha, A, lda, x, incx, beta, y, incy, layout)


def check_factor(oracle, routine, got, a):
    want = oracle.gemv(*a)
    f = oracle.gemv_forward_factor(got, want, *a)
    assert f <= THRESHOLD[routine], f
    trans, m, n = a[0], a[1], a[2]
    ylen = m if trans == "no-transpose" else n
    gaps = np.ones(got.size, bool)
    gaps[np.arange(ylen) * a[10]] = False
    assert bits_equal(got[gaps], a[9][gaps]), "a gap of the strided y changed"


@pytest.mark.parametrize("routine", ["sgemv", "dgemv"])
def test_fixtures(wg, device, oracle, routine):
    """Seeded random cases in the reference's fixture ranges (m, n <= 50, any
    trans, layout, stride, padded lda, alpha and beta)."""
    rng = np.random.default_rng(100)
    dt = dtype_of(routine)
    for seed in range(40):
        trans = ("no-transpose", "transpose")[seed % 2]
        layout = ("row-major", "column-major")[(seed // 2) % 2]
        m, n = int(rng.integers(1, 51)), int(rng.integers(1, 51))
        incx, incy = int(rng.integers(1, 5)), int(rng.integers(1, 5))
        alpha, beta = float(rng.choice([0.0, 1.0, -1.0, 0.5, 2.5])), float(rng.choice([0.0, 1.0, -1.0, 0.25]))
        a = random_case(dt, trans, layout, m, n, incx, incy, seed, alpha, beta, pad=int(rng.integers(0, 3)))
        check_factor(oracle, routine, call(wg, device, routine, a)["y"], a)


@pytest.mark.parametrize("routine", ["sgemv", "dgemv"])
def test_zero_contraction_dimension_leaves_y(wg, device, routine):
    dt = dtype_of(routine)
    fn = getattr(wg, routine)
    for trans, m, n in (("no-transpose", 4, 0), ("transpose", 0, 4)):
        y = wg.randomFloat64Array(4, -1, 1, 9001).astype(dt)
        before = y.copy()
        got = fn(device, trans, m, n, 1.5, np.zeros(0, dt), 1, np.zeros(0, dt), 1, 0.5, y, 1)["y"]
        assert bits_equal(got, before)


@pytest.mark.parametrize("routine", ["sgemv", "dgemv"])
@pytest.mark.parametrize("layout,trans", [("row-major", "transpose"), ("column-major", "no-transpose"),
                                          ("row-major", "no-transpose"), ("column-major", "transpose")])
@pytest.mark.parametrize("beta", [0.0, 0.75])
@pytest.mark.parametrize("inc", [1, 3])
def test_split_chunks(wg, device, oracle, routine, layout, trans, beta, inc):
    """600 x 300 (test.sgemv.js:204-256): several row or column chunks summed by
    the second kernel, beta = 0 and not, strided x and y."""
    m, n = (600, 300) if layout == "row-major" else (300, 600)
    a = random_case(dtype_of(routine), trans, layout, m, n, inc, inc, 21, beta=beta)
    check_factor(oracle, routine, call(wg, device, routine, a)["y"], a)


@pytest.mark.parametrize("n,m,inc,beta", [(600, 70, 1, 0.75), (600, 70, 2, 0.75), (600, 70, 1, 0.0),
                                          (256, 33, 1, 0.75), (319, 33, 3, 0.75)])
def test_dgemv_long_rows(wg, device, oracle, n, m, inc, beta):
    """test.dgemv.js:285-342: row-major no-transpose with long rows and lda = n + 3."""
    a = random_case(np.float64, "no-transpose", "row-major", m, n, inc, inc, 31, beta=beta, pad=3)
    check_factor(oracle, "dgemv", call(wg, device, "dgemv", a)["y"], a)


def at(n, r, c):
    return r * n + c


def assert_ieee_match(got, want, tol):
    g, w = np.asarray(got, np.float64), np.asarray(want, np.float64)
    nan = np.isnan(w)
    assert np.all(np.isnan(g[nan])), "NaN expected"
    inf = np.isinf(w)
    assert np.all(g[inf] == w[inf]), "signed Infinity expected"
    fin = ~nan & ~inf
    assert np.all(np.isfinite(g[fin]))
    assert np.all(np.abs(g[fin] - w[fin]) <= tol * np.maximum(1.0, np.abs(w[fin])))


@pytest.mark.parametrize("routine", ["sgemv", "dgemv"])
@pytest.mark.parametrize("trans", ["no-transpose", "transpose"])
@pytest.mark.parametrize("n", [7, 300])
@pytest.mark.parametrize("beta", [0.0, 0.5])
def test_alpha_zero_reads_neither_a_nor_x(wg, device, oracle, routine, trans, n, beta):
    dt = dtype_of(routine)
    A = wg.randomFloat64Array(n * n, -1, 1, 1).astype(dt)
    A[at(n, 1, 2)] = np.nan
    A[at(n, 3, 4)] = np.inf
    x = wg.randomFloat64Array(n, -1, 1, 2).astype(dt)
    x[5] = -np.inf
    y = wg.randomFloat64Array(n, -1, 1, 3).astype(dt)
    if beta == 0:
        y[0] = np.nan
    a = (trans, n, n, 0.0, A, n, x, 1, beta, y, 1, "row-major")
    assert_ieee_match(call(wg, device, routine, a)["y"], oracle.gemv(*a), 1e-4)


@pytest.mark.parametrize("routine", ["sgemv", "dgemv"])
@pytest.mark.parametrize("layout", ["row-major", "column-major"])
@pytest.mark.parametrize("trans", ["no-transpose", "transpose"])
@pytest.mark.parametrize("n", [7, 300])
def test_zero_x_entries_skip_their_column(wg, device, oracle, routine, layout, trans, n):
    """test.sgemv.js:341-386: the column form (row-major transpose, column-major
    no-transpose) skips a column whose x entry is 0; the dot form takes 0 * Infinity."""
    dt = dtype_of(routine)
    A = wg.randomFloat64Array(n * n, -1, 1, 1).astype(dt)
    A[at(n, 1, 2)] = np.inf
    A[at(n, 2, 1)] = -np.inf
    A[at(n, 4, 0)] = np.nan
    A[at(n, 0, 4)] = np.inf
    x = wg.randomFloat64Array(n, -1, 1, 2).astype(dt)
    x[1] = 0
    x[4] = 0
    y = wg.randomFloat64Array(n, -1, 1, 3).astype(dt)
    a = (trans, n, n, 1.5, A, n, x, 1, 0.5, y, 1, layout)
    assert_ieee_match(call(wg, device, routine, a)["y"], oracle.gemv(*a), 1e-4)


@pytest.mark.parametrize("trans", ["no-transpose", "transpose"])
@pytest.mark.parametrize("n", [7, 300])
def test_dgemv_ieee_special_values(wg, device, oracle, trans, n):
    """test.dgemv.js:430-476: Infinity and NaN reach y as real f64 puts them;
    beta = 0 ignores NaN and Infinity already in y."""
    A = wg.randomFloat64Array(n * n, -1, 1, 1)
    A[at(n, 1, 2)] = np.inf
    A[at(n, 3, 4)] = np.nan
    x = wg.randomFloat64Array(n, -1, 1, 2)
    x[5] = -np.inf
    y = wg.randomFloat64Array(n, -1, 1, 3)
    y[0] = np.nan
    y[6] = np.inf
    a = (trans, n, n, 1.5, A, n, x, 1, 0.0, y, 1, "row-major")
    want = oracle.gemv(*a[:9], np.zeros(n), *a[10:])
    assert_ieee_match(call(wg, device, "dgemv", a)["y"], want, 1e-12)


def test_dgemv_exactness(wg, device):
    """test.dgemv.js:383-428: alpha = 0 with beta = 1 returns the given y itself;
    strided gaps of y come back bit-identical."""
    rng = np.random.default_rng(960)
    n = 5
    for trans in ("no-transpose", "transpose"):
        y = rng.random(n) * np.pi
        r = wg.dgemv(device, trans, n, n, 0.0, rng.random(n * n), n, rng.random(n), 1, 1.0, y, 1)
        assert r["y"] is y
    for beta in (0.0, 0.5):
        y = rng.random(13) * np.pi
        got = wg.dgemv(device, "no-transpose", n, n, 1.5, rng.random(n * n), n, rng.random(13), 3, beta, y, 3)["y"]
        gaps = np.ones(13, bool)
        gaps[np.arange(n) * 3] = False
        assert bits_equal(got[gaps], y[gaps])


def test_dgemv_keeps_the_f64_exponent_range(wg, device, oracle):
    """Native fp64 (an intended divergence: the reference's double-double reads
    values beyond f32's range as Infinity or 0, test.dgemv.js:478-551)."""
    n = 7
    A = np.full(n * n, 1e200)
    x = np.full(n, 1e100)
    y = np.full(n, 1e-300)
    for trans in ("no-transpose", "transpose"):
        a = (trans, n, n, 1e-250, A, n, x, 1, 0.5, y, 1, "row-major")
        got = call(wg, device, "dgemv", a)["y"]
        assert np.all(np.isfinite(got)) and np.allclose(got, oracle.gemv(*a), rtol=1e-14)


@pytest.mark.parametrize("routine", ["sgemv", "dgemv"])
@pytest.mark.parametrize("layout", ["row-major", "column-major"])
def test_gpu_operands_in_place(wg, device, oracle, routine, layout):
    dt = dtype_of(routine)
    m, n = 257, 130
    for trans in ("no-transpose", "transpose"):
        a = random_case(dt, trans, layout, m, n, 1, 1, 41, pad=3)
        _, _, _, alpha, A, lda, x, incx, beta, y, incy, _ = a
        GA = wg.GpuMatrix.from_(device, A, m, n, lda, layout)
        gx, gy = wg.GpuVector.from_(device, x), wg.GpuVector.from_(device, y)
        try:
            r = getattr(wg, routine)(device, trans, m, n, alpha, GA, lda, gx, incx, beta, gy, incy)
            assert "y" not in r
            got = gy.read()
            with pytest.raises(wg.Error, match="must not reference the same GPU buffer"):
                getattr(wg, routine)(device, trans, m, n, alpha, GA, lda, gy, incx, beta, gy, incy)
        finally:
            GA.destroy()
            gx.destroy()
            gy.destroy()
        check_factor(oracle, routine, got, a)


@pytest.mark.parametrize("routine", ["sgemv", "dgemv"])
@pytest.mark.parametrize("trans", ["no-transpose", "transpose"])
def test_full_size(wg, device, oracle, routine, trans):
    """4096 x 4096, column-major (the reference's base sweep layout): both kernels."""
    a = random_case(dtype_of(routine), trans, "column-major", 4096, 4096, 1, 1, 51)
    check_factor(oracle, routine, call(wg, device, routine, a)["y"], a)


@pytest.mark.parametrize("routine", ["sgemv", "dgemv"])
@pytest.mark.parametrize("m,n,pad", [(2371, 37, 1), (4099, 130, 1), (9000, 20, 0), (30001, 9, 3)])
@pytest.mark.parametrize("beta,inc", [(0.0, 1), (0.75, 1), (0.75, 3)])
def test_row_blocks(wg, device, oracle, routine, m, n, pad, beta, inc):
    """Column-major no-transpose with enough rows for one CTA per row block over
    every column: a ragged last block, a last vector that crosses row m (read
    one element at a time, the host copy ends at row m of the last column),
    padded lda, segments of 4, 8 and 32 lanes, unit and strided x and y."""
    a = random_case(dtype_of(routine), "no-transpose", "column-major", m, n, inc, inc, m + n, beta=beta, pad=pad)
    check_factor(oracle, routine, call(wg, device, routine, a)["y"], a)


@pytest.mark.parametrize("routine", ["sgemv", "dgemv"])
def test_row_blocks_zero_x_skips_its_column(wg, device, oracle, routine):
    """The row-block kernel loads every column but adds nothing for a zero x
    entry, so Infinity and NaN there never reach y; elsewhere they do."""
    m, n = 4099, 64
    a = list(random_case(dtype_of(routine), "no-transpose", "column-major", m, n, 1, 1, 5, beta=0.0, pad=1))
    A, lda, x, y = a[4], a[5], a[6], a[9]
    for j in (0, 17, 63):
        x[j] = 0
        A[j * lda:j * lda + m:5] = np.nan
        A[j * lda + m - 1] = np.inf
    A[3 * lda + 100] = -np.inf
    A[40 * lda + m - 2] = np.nan
    y[7] = np.nan  # beta = 0: y is not read
    assert_ieee_match(call(wg, device, routine, tuple(a))["y"], oracle.gemv(*a), 1e-4)
