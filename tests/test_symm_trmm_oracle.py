"""ssymm/dsymm and strmm/dtrmm golden edge cases (tests/golden/symm_trmm_edge_cases.json,
from the reference's tests/{s,d}{symm,trmm}/edge-cases*.json with exact expected
results) reproduced bit for bit by the oracle's restatement of the reference's
algorithm: a dense copy of the symmetric / triangular operand (symmetrize.wgsl,
triangularize.wgsl) followed by the GEMM arithmetic (src/ssymm/ssymm.mjs:26-28,
src/strmm/strmm.mjs). CPU only."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import bits_equal, load_golden


def elem(M, ld, layout, r, c):
    return M[c * ld + r] if layout == "column-major" else M[r * ld + c]


def dense_operand(case, dt):
    """The order x order operand the GEMM sees, column-major: A symmetrized (symm)
    or op(A) triangularized (trmm)."""
    lay, m, n = case["layout"], case["m"], case["n"]
    order = m if case["side"] == "left" else n
    lower = case["uplo"] == "lower"
    trmm = case["routine"].endswith("trmm")
    D = np.zeros(order * order, dt)
    for j in range(order):
        for i in range(order):
            if trmm:
                r, c = (j, i) if case["transA"] == "transpose" else (i, j)
                if r == c:
                    v = 1.0 if case["diag"] == "unit" else elem(case["A"], case["lda"], lay, r, r)
                else:
                    v = elem(case["A"], case["lda"], lay, r, c) if (r > c if lower else r < c) else 0.0
            else:
                stored = i >= j if lower else i <= j
                v = elem(case["A"], case["lda"], lay, i, j) if stored else elem(case["A"], case["lda"], lay, j, i)
            D[i + j * order] = v
    return D, order


def general(case, name, ld, dt):
    lay, m, n = case["layout"], case["m"], case["n"]
    return np.array([elem(case[name], ld, lay, i, j) for j in range(n) for i in range(m)], dt)


def restate(oracle, case, variant):
    f64 = case["routine"].startswith("d")
    dt = np.float64 if f64 else np.float32
    m, n = case["m"], case["n"]
    trmm = case["routine"].endswith("trmm")
    D, order = dense_operand(case, dt)
    Bd = general(case, "B", case["ldb"], dt)
    Cd = np.zeros(m * n, dt) if trmm else general(case, "C", case["ldc"], dt)
    beta = 0.0 if trmm else case["beta"]
    X, ldx, Y, ldy = (D, order, Bd, m) if case["side"] == "left" else (Bd, m, D, order)
    if f64:
        res = oracle.dgemm_fma(0, 0, m, n, order, case["alpha"], X, ldx, Y, ldy, beta, Cd, m)
    else:
        res = oracle.sgemm(0, 0, m, n, order, case["alpha"], X, ldx, Y, ldy, beta, Cd, m, variant=variant)
    name, ld = ("B", case["ldb"]) if trmm else ("C", case["ldc"])
    out = np.array(case[name], dt)
    for j in range(n):
        for i in range(m):
            out[(j * ld + i) if case["layout"] == "column-major" else (i * ld + j)] = res[i + j * m]
    return out


@pytest.mark.parametrize("case", load_golden("symm_trmm_edge_cases.json"),
                         ids=lambda c: f"{c['routine']}:{c['label'][:40]}")
def test_symm_trmm_edge_cases_exact(oracle, case):
    dt = np.float64 if case["routine"].startswith("d") else np.float32
    want = np.array(case["expected"], dt)
    for variant in (0, 1):
        assert bits_equal(restate(oracle, case, variant), want), case["label"]


def test_golden_covers_the_reference_files():
    by = {}
    for c in load_golden("symm_trmm_edge_cases.json"):
        by[c["routine"]] = by.get(c["routine"], 0) + 1
    assert by == {"ssymm": 14, "dsymm": 15, "strmm": 14, "dtrmm": 18}
