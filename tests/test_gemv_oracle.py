"""The gemv oracle (oracle.gemv, a restatement of reference BLAS xGEMV as the
reference's tests call it through stdlib, and oracle.gemv_forward_factor, its
tests/{sgemv,dgemv}/helpers.js) pinned on CPU: the reference's 28 edge cases
bit for bit against exact rational results (tests/golden/gemv_edge_cases.json),
random cases against an fp64 product, and the zero-x and alpha = 0 rules."""
from __future__ import annotations

import math

import numpy as np
import pytest

from conftest import bits_equal, load_golden

CASES = load_golden("gemv_edge_cases.json")


def args(case, dt):
    return (case["trans"], case["m"], case["n"], case["alpha"], np.array(case["A"], dt), case["lda"],
            np.array(case["x"], dt), case["incx"], case["beta"], np.array(case["y"], dt), case["incy"],
            case["layout"])


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"{c['routine']}:{c['label'][:40]}")
def test_edge_cases_exact(oracle, case):
    dt = np.float64 if case["routine"] == "dgemv" else np.float32
    got = oracle.gemv(*args(case, dt))
    assert bits_equal(got, np.array(case["expected"], dt)), (got, case["expected"])


def random_case(dt, trans, layout, m, n, inc, seed, alpha=1.25, beta=-0.5):
    rng = np.random.default_rng(seed)
    cm = layout == "column-major"
    lda = (m if cm else n) + 2
    A = (rng.random(lda * (n if cm else m)) * 2 - 1).astype(dt)
    no_t = trans == "no-transpose"
    xlen, ylen = (n, m) if no_t else (m, n)
    x = (rng.random((xlen - 1) * inc + 1) * 2 - 1).astype(dt)
    y = (rng.random((ylen - 1) * inc + 1) * 2 - 1).astype(dt)
    return (trans, m, n, alpha, A, lda, x, inc, beta, y, inc, layout)


def fp64_truth(a):
    trans, m, n, alpha, A, lda, x, incx, beta, y, incy, layout = a
    cm = layout == "column-major"
    M = (A.reshape(-1, lda).T if cm else A.reshape(-1, lda))[:m, :n].astype(np.float64)
    op = M if trans == "no-transpose" else M.T
    xv = x[np.arange(op.shape[1]) * incx].astype(np.float64)
    iy = np.arange(op.shape[0]) * incy
    out = y.astype(np.float64).copy()
    out[iy] = alpha * (op @ xv) + beta * out[iy]
    return out


@pytest.mark.parametrize("dt", [np.float32, np.float64])
@pytest.mark.parametrize("trans", ["no-transpose", "transpose"])
@pytest.mark.parametrize("layout", ["row-major", "column-major"])
def test_random_against_fp64(oracle, dt, trans, layout):
    a = random_case(dt, trans, layout, 37, 53, 2, seed=3)
    got = oracle.gemv(*a)
    truth = fp64_truth(a)
    f = oracle.gemv_forward_factor(got, truth.astype(dt), *a)
    assert f <= 4.0, f
    gaps = np.ones(got.size, bool)
    gaps[np.arange(37 if trans == "no-transpose" else 53) * 2] = False
    assert bits_equal(got[gaps], a[9][gaps])


def test_zero_x_columns_are_skipped_only_in_the_column_form(oracle):
    n = 7
    A = np.ones(n * n, np.float32)
    A[1 * n + 2] = np.inf  # row 1, col 2 (row-major)
    x = np.ones(n, np.float32)
    x[2] = 0.0
    y = np.zeros(n, np.float32)
    # Row-major transpose runs column by column over A's rows (A^T x contracts
    # over them): x[1] = 1 multiplies row 1, x[2] = 0 skips row 2.
    t = oracle.gemv("transpose", n, n, 1.0, A, n, x, 1, 0.0, y, 1)
    assert np.isinf(t[2])  # row 1 (x[1] = 1) carries the Infinity into y[2]
    x2 = np.ones(n, np.float32)
    x2[1] = 0.0
    t2 = oracle.gemv("transpose", n, n, 1.0, A, n, x2, 1, 0.0, y, 1)
    assert np.all(np.isfinite(t2))  # row 1 skipped: no 0 * Infinity
    # row-major no-transpose is the dot-product form: 0 * Infinity = NaN
    nt = oracle.gemv("no-transpose", n, n, 1.0, A, n, x, 1, 0.0, y, 1)
    assert math.isnan(nt[1])


def test_alpha_zero_reads_neither_a_nor_x(oracle):
    n = 5
    A = np.full(n * n, np.nan, np.float32)
    x = np.full(n, np.inf, np.float32)
    y = np.array([np.nan, 1, 2, 3, 4], np.float32)
    z = oracle.gemv("no-transpose", n, n, 0.0, A, n, x, 1, 0.0, y, 1)
    assert bits_equal(z, np.zeros(n, np.float32))
    half = oracle.gemv("transpose", n, n, 0.0, A, n, x, 1, 0.5, np.arange(n, dtype=np.float32), 1)
    assert bits_equal(half, np.arange(n, dtype=np.float32) * np.float32(0.5))
    same = oracle.gemv("transpose", n, n, 0.0, A, n, x, 1, 1.0, y, 1)
    assert bits_equal(same, y)


def test_forward_factor_flags_a_wrong_result(oracle):
    a = random_case(np.float32, "no-transpose", "row-major", 20, 30, 1, seed=4)
    good = oracle.gemv(*a)
    truth = fp64_truth(a).astype(np.float32)
    assert oracle.gemv_forward_factor(good, truth, *a) <= 4.0
    bad = good.copy()
    bad[3] *= np.float32(1.0001)
    assert oracle.gemv_forward_factor(bad, truth, *a) > 4.0
