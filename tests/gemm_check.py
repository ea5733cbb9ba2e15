"""Shared parity checks of GPU sgemm/dgemm results against the CPU oracle.

Bounds used (all written here, per element of the m x n block):
* sgemm, north star: |got - x| <= 2*K*2^-24*(|alpha|sum|a||b| + |beta||c|) for x the
  fp64 truth and for x the oracle's restatement of the reference's fp32 arithmetic;
* sgemm, the reference's own forwardFactor (tests/sgemm/helpers.js, eps=2^-23,
  (k+1)|alpha|, |beta|) against the fp64 truth: <= 1;
* dgemm, north star: |got - truth| <= 4*K*2^-53*(|alpha|sum|a||b| + |beta||c|);
* elements outside the m x n block (leading-dimension padding) are unchanged.
"""
from __future__ import annotations

import numpy as np

from conftest import bits_equal


def frame(transA, transB, m, n, A, lda, B, ldb, layout):
    """Column-major-frame arguments (an independent copy of the mapping under test)."""
    cm = layout == "column-major"
    ta = (transA == "transpose") == cm
    tb = (transB == "transpose") == cm
    if cm:
        return int(ta), int(tb), m, n, A, lda, B, ldb
    return int(not tb), int(not ta), n, m, B, ldb, A, lda


def block_mask(size, m_rows, n_cols, ld):
    """True on the elements of the column-major m_rows x n_cols block."""
    mask = np.zeros(size, bool)
    for j in range(n_cols):
        mask[j * ld: j * ld + m_rows] = True
    return mask


def check_sgemm(oracle, got, transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc,
                layout="row-major", exact=False):
    """Returns a dict of measured deviations; asserts every bound."""
    alpha = float(np.float32(alpha))
    beta = float(np.float32(beta))
    ta, tb, mm, nn, AA, l1, BB, l2 = frame(transA, transB, m, n, A, lda, B, ldb, layout)
    ref = oracle.sgemm(ta, tb, mm, nn, k, alpha, AA, l1, BB, l2, beta, C, ldc, variant=1)
    truth, absab = oracle.sgemm_truth(ta, tb, mm, nn, k, alpha, AA, l1, BB, l2, beta, C, ldc)
    g = oracle.block(got, mm, nn, ldc).astype(np.float64)
    r = oracle.block(ref, mm, nn, ldc).astype(np.float64)
    t = oracle.dense(truth, mm, nn)
    bound = oracle.sgemm_bound(mm, nn, k, alpha, absab, beta, C, ldc)
    finite = np.isfinite(t)
    e_truth = np.abs(g - t)[finite]
    e_ref = np.abs(g - r)[finite]
    assert np.all(e_truth <= bound[finite]), f"max excess vs truth {np.max(e_truth - bound[finite])}"
    assert np.all(e_ref <= bound[finite]), f"max excess vs restatement {np.max(e_ref - bound[finite])}"
    ff = oracle.forward_factor(np.where(np.isfinite(got), got, 0).astype(np.float32), truth, mm, nn, k,
                               alpha, absab, beta, C, ldc, 2.0**-23, 1, 1) if np.all(finite) else 0.0
    assert ff <= 1, f"reference forward factor {ff}"
    outside = ~block_mask(C.size, mm, nn, ldc)
    assert bits_equal(got[outside], C[outside]), "padding of C was written"
    if exact:
        assert bits_equal(got, ref), "not bit-identical to the FMA restatement"
    return {"forward_factor": ff,
            "max_bound_frac": float(np.max(e_truth / np.where(bound[finite] > 0, bound[finite], 1)))
            if e_truth.size else 0.0,
            "max_abs_vs_restatement": float(np.max(e_ref)) if e_ref.size else 0.0}


def check_dgemm(oracle, got, transA, transB, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc,
                layout="row-major", exact=False):
    ta, tb, mm, nn, AA, l1, BB, l2 = frame(transA, transB, m, n, A, lda, B, ldb, layout)
    truth, absab = oracle.dgemm_truth(ta, tb, mm, nn, k, alpha, AA, l1, BB, l2, beta, C, ldc)
    g = oracle.block(got, mm, nn, ldc)
    t = oracle.dense(truth, mm, nn)
    bound = oracle.dgemm_bound(mm, nn, k, alpha, absab, beta, C, ldc)
    finite = np.isfinite(t)
    err = np.abs(g - t)[finite]
    assert np.all(err <= bound[finite]), f"max excess vs truth {np.max(err - bound[finite])}"
    outside = ~block_mask(C.size, mm, nn, ldc)
    assert bits_equal(got[outside], C[outside]), "padding of C was written"
    if exact:
        fm = oracle.dgemm_fma(ta, tb, mm, nn, k, alpha, AA, l1, BB, l2, beta, C, ldc)
        assert bits_equal(got, fm), "not bit-identical to the fp64 FMA restatement"
    dd = oracle.dgemm_dd(ta, tb, mm, nn, k, alpha, AA, l1, BB, l2, beta, C, ldc)
    dd_err = np.abs(oracle.block(dd, mm, nn, ldc) - t)[finite]
    return {"max_bound_frac": float(np.max(err / np.where(bound[finite] > 0, bound[finite], 1)))
            if err.size else 0.0,
            "reference_dd_max_abs_err": float(np.max(dd_err)) if dd_err.size else 0.0,
            "ours_max_abs_err": float(np.max(err)) if err.size else 0.0}


def ieee_match(got, want, tol):
    """assertIeeeMatch (tests/helpers/specials.js:23-40): NaN<->NaN, the same signed
    Infinity, finite within tol relative (floor tol)."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    assert got.shape == want.shape
    nan = np.isnan(want)
    assert np.all(np.isnan(got[nan])), "NaN expected"
    inf = np.isinf(want)
    assert np.array_equal(got[inf], want[inf]), "Infinity mismatch"
    fin = ~nan & ~inf
    assert np.all(np.isfinite(got[fin]))
    assert np.all(np.abs(got[fin] - want[fin]) <= tol * np.maximum(1, np.abs(want[fin])))


def fixture_args(rng, f64):
    """One random case shaped like the reference's fast-check fixtures
    (tests/helpers/fixtures.js: m, n, k in [1, 20], random trans and layout, ld at or
    above its minimum, scalars and elements in [-10, 10] with |x| >= 1e-3 or 0)."""
    dt = np.float64 if f64 else np.float32
    m, n, k = (int(x) for x in rng.integers(1, 21, 3))
    transA = ("no-transpose", "transpose")[int(rng.integers(0, 2))]
    transB = ("no-transpose", "transpose")[int(rng.integers(0, 2))]
    layout = ("row-major", "column-major")[int(rng.integers(0, 2))]
    cm = layout == "column-major"
    a_rows, a_cols = (m, k) if transA == "no-transpose" else (k, m)
    b_rows, b_cols = (k, n) if transB == "no-transpose" else (n, k)
    lda = (a_rows if cm else a_cols) + int(rng.integers(0, 3))
    ldb = (b_rows if cm else b_cols) + int(rng.integers(0, 3))
    ldc = (m if cm else n) + int(rng.integers(0, 3))

    def vals(size):
        v = rng.uniform(-10, 10, size)
        v[np.abs(v) < 1e-3] = 0
        return v.astype(dt)

    def scalar():
        v = float(rng.uniform(-10, 10))
        return 0.0 if abs(v) < 1e-3 else v

    A = vals(lda * (a_cols if cm else a_rows))
    B = vals(ldb * (b_cols if cm else b_rows))
    C = vals(ldc * (n if cm else m))
    return dict(transA=transA, transB=transB, m=m, n=n, k=k, alpha=scalar(), A=A, lda=lda, B=B,
                ldb=ldb, beta=scalar(), C=C, ldc=ldc, layout=layout)


def sampled_columns_truth(oracle, f64, ta, tb, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc, cols):
    """fp64/long-double truth and sum|a||b| for a subset of C's columns (column-major frame),
    so a full-size result can be checked without a full CPU GEMM."""
    dt = np.float64 if f64 else np.float32
    opB = np.empty((k, len(cols)), dt)
    for c, j in enumerate(cols):
        opB[:, c] = B[j + np.arange(k) * ldb] if tb else B[j * ldb: j * ldb + k]
    Bs = np.ascontiguousarray(opB.T).reshape(-1)  # column-major k x len(cols), ld = k
    Cs = np.empty(m * len(cols), dt)
    for c, j in enumerate(cols):
        Cs[c * m:(c + 1) * m] = C[j * ldc: j * ldc + m]
    fn = oracle.dgemm_truth if f64 else oracle.sgemm_truth
    truth, absab = fn(ta, 0, m, len(cols), k, alpha, A, lda, Bs, max(k, 1), beta, Cs, m)
    return truth, absab, Cs
