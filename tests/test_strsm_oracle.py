"""The strsm oracle (oracle.strsm, a restatement of the reference's own test
oracle, tests/helpers/stdlib.js:607-775, and oracle.strsm_residual_factor, its
tests/strsm/helpers.js) pinned before the GPU tests rely on it: the reference's
edge cases against their exact rational solutions (tests/golden/strsm_edge_cases.json),
random systems against an independent fp64 solver, and the IEEE rules the
reference's strsm tests check. CPU only."""
from __future__ import annotations

import math

import numpy as np
import pytest
from scipy.linalg import solve_triangular

from conftest import bits_equal, load_golden

CASES = load_golden("strsm_edge_cases.json")


def args(case, B=None):
    return (case["side"], case["uplo"], case["transA"], case["diag"], case["m"], case["n"], case["alpha"],
            np.array(case["A"], np.float32), case["lda"], np.array(case["B"] if B is None else B, np.float32),
            case["ldb"], case["layout"])


@pytest.mark.parametrize("case", CASES, ids=lambda c: c["label"][:50])
def test_edge_cases_match_exact_solutions(oracle, case):
    got = oracle.strsm(*args(case))
    want = np.array(case["expected"], np.float32)
    if case["exact"]:
        assert bits_equal(got, want), (got, want)
    else:
        # The substitution stores every unknown rounded to f32 before the next
        # one uses it, so inexact solutions differ from the exact one by a few ulps.
        assert np.allclose(got, want, rtol=2.0**-20, atol=0), (got, want)
    factor = oracle.strsm_residual_factor(got, *args(case))
    assert factor <= (0.0 if case["exact"] else 5.0), factor


def test_edge_case_inventory():
    assert len(CASES) == 14
    assert {c["layout"] for c in CASES} == {"row-major", "column-major"}
    assert {(c["side"], c["uplo"]) for c in CASES} == {("left", "lower"), ("left", "upper"), ("right", "lower"),
                                                       ("right", "upper")}


def system(side, uplo, transA, diag, layout, m, n, pad, seed):
    """A well-conditioned case: off-diagonals of +-1/order, diagonal 2 (tests/strsm/src/test.strsm.js:344-352)."""
    rng = np.random.default_rng(seed)
    order = m if side == "left" else n
    cm = layout == "column-major"
    A = ((rng.random(order * order) * 2 - 1) / order).astype(np.float32)
    A[np.arange(order) * (order + 1)] = 2.0
    ldb = (m if cm else n) + pad
    B = (rng.random(ldb * (n if cm else m)) * 2 - 1).astype(np.float32)
    return (side, uplo, transA, diag, m, n, 1.5, A, order, B, ldb, layout)


def scipy_solution(a):
    side, uplo, transA, diag, m, n, alpha, A, lda, B, ldb, layout = a
    order = m if side == "left" else n
    cm = layout == "column-major"
    M = (A.reshape(order, lda).T if cm else A.reshape(order, lda))[:, :order].astype(np.float64)
    M = np.tril(M) if uplo == "lower" else np.triu(M)
    if diag == "unit":
        np.fill_diagonal(M, 1.0)
    op = M.T if transA == "transpose" else M
    idx = (np.arange(n)[None, :] * ldb + np.arange(m)[:, None]) if cm else \
        (np.arange(m)[:, None] * ldb + np.arange(n)[None, :])
    rhs = alpha * B[idx].astype(np.float64)
    low = np.allclose(op, np.tril(op))
    if side == "left":
        return solve_triangular(op, rhs, lower=low), idx
    return solve_triangular(op.T, rhs.T, lower=not low).T, idx


@pytest.mark.parametrize("side", ["left", "right"])
@pytest.mark.parametrize("uplo", ["lower", "upper"])
@pytest.mark.parametrize("transA", ["no-transpose", "transpose"])
@pytest.mark.parametrize("layout", ["row-major", "column-major"])
def test_against_fp64_solver(oracle, side, uplo, transA, layout):
    diag = "unit" if transA == "transpose" else "non-unit"
    a = system(side, uplo, transA, diag, layout, m=23 if side == "left" else 9, n=9 if side == "left" else 23, pad=2,
               seed=(side == "left") * 8 + (uplo == "lower") * 4 + (transA == "transpose") * 2 + (layout == "row-major"))
    got = oracle.strsm(*a)
    want, idx = scipy_solution(a)
    assert np.allclose(got[idx], want, rtol=1e-5, atol=1e-6)
    pad = np.ones(got.size, bool)
    pad[idx.ravel()] = False
    assert bits_equal(got[pad], a[9][pad])
    assert oracle.strsm_residual_factor(got, *a) <= 1.0


def test_ieee_rules(oracle):
    """Infinity in B spreads along the substitution, NaN in the unreferenced
    triangle is never read, alpha = 0 gives zeros (tests/strsm/src/test.strsm.js:166-198,498-578)."""
    m, n = 7, 5
    rng = np.random.default_rng(3)
    A = (rng.random(m * m) * 2 - 1).astype(np.float32)
    A[np.arange(m) * (m + 1)] += m + 4
    A[1 * m + 4] = np.nan  # row 1, col 4: above the diagonal, unreferenced for 'lower'
    B = (rng.random(m * n) * 2 - 1).astype(np.float32)
    X = oracle.strsm("left", "lower", "no-transpose", "non-unit", m, n, 1.0, A, m, B, n)
    assert np.all(np.isfinite(X))
    B2 = B.copy()
    B2[1 * n + 2] = np.inf
    X2 = oracle.strsm("left", "lower", "no-transpose", "non-unit", m, n, 1.0, A, m, B2, n)
    col = X2.reshape(m, n)[:, 2]
    assert np.all(np.isfinite(col[:1])) and not np.any(np.isfinite(col[1:]))
    assert np.all(np.isfinite(np.delete(X2.reshape(m, n), 2, axis=1)))
    poisoned = np.array([math.inf, math.nan, 3, 4], np.float32)
    z = oracle.strsm("left", "lower", "no-transpose", "non-unit", 2, 2, 0.0, np.array([1, 0, 1, 1], np.float32), 2,
                     poisoned, 2)
    assert bits_equal(z, np.zeros(4, np.float32))


def test_zero_dimensions_return_b_unchanged(oracle):
    B = np.arange(16, dtype=np.float32)
    for m, n in ((0, 4), (4, 0)):
        got = oracle.strsm("left", "lower", "no-transpose", "non-unit", m, n, 1.5, np.zeros(0, np.float32), 1, B, 4)
        assert bits_equal(got, B)


def test_residual_factor_flags_a_wrong_solution(oracle):
    a = system("left", "lower", "no-transpose", "non-unit", "row-major", 12, 6, 0, 5)
    X = oracle.strsm(*a)
    bad = X.copy()
    bad[7] = np.nextafter(np.nextafter(bad[7], np.float32(np.inf)), np.float32(np.inf)) * np.float32(1.001)
    assert oracle.strsm_residual_factor(X, *a) <= 1.0
    assert oracle.strsm_residual_factor(bad, *a) > 5.0
