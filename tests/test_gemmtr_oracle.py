"""The gemmtr family's golden edge cases (tests/golden/gemmtr_edge_cases.json,
from the reference's tests/{s,d}{gemmtr,syrk,syr2k}/edge-cases*.json with exact
expected results) reproduced bit for bit by the oracle's restatement: gemmtr is
sgemm's per-element arithmetic written only in the uplo triangle; syrk is gemmtr
with B := A and the other transpose; syr2k two gemmtr passes, the second with
beta = 1 (src/ssyrk/ssyrk.mjs:29-31, src/ssyr2k/ssyr2k.mjs:25-26). CPU only."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import bits_equal, load_golden

FLIP = {"transpose": "no-transpose", "no-transpose": "transpose"}


def as_gemmtr_passes(case):
    """The case as one or two gemmtr calls in the user's terms (routine, A, lda, B, ldb, beta)."""
    r = case["routine"][1:]
    if r == "gemmtr":
        return [(case["transA"], case["transB"], case["m"], case["A"], case["lda"], case["B"], case["ldb"],
                 case["beta"])]
    t, ft, n = case["trans"], FLIP[case["trans"]], case["n"]
    if r == "syrk":
        return [(t, ft, n, case["A"], case["lda"], case["A"], case["lda"], case["beta"])]
    return [(t, ft, n, case["A"], case["lda"], case["B"], case["ldb"], case["beta"]),
            (t, ft, n, case["B"], case["ldb"], case["A"], case["lda"], 1.0)]


def run_gemmtr(fn, dt, case, tA, tB, m, A, lda, B, ldb, beta, C):
    """One gemmtr call through the column-major frame (the row-major twin swaps
    operands, m/n and the triangle)."""
    n, k = case["n"], case["k"]
    cm = case["layout"] == "column-major"
    ta = (tA == "transpose") == cm
    tb = (tB == "transpose") == cm
    uplo = 1 if case["uplo"] == "lower" else 2
    A = np.array(A, dt)
    B = np.array(B, dt)
    if cm:
        return fn(uplo, int(ta), int(tb), m, n, k, case["alpha"], A, lda, B, ldb, beta, C, case["ldc"])
    return fn(3 - uplo, int(not tb), int(not ta), n, m, k, case["alpha"], B, ldb, A, lda, beta, C, case["ldc"])


@pytest.mark.parametrize("case", load_golden("gemmtr_edge_cases.json"),
                         ids=lambda c: f"{c['routine']}:{c['label'][:40]}")
def test_gemmtr_family_edge_cases_exact(oracle, case):
    f64 = case["routine"].startswith("d")
    dt = np.float64 if f64 else np.float32
    fns = [oracle.dgemmtr_fma] if f64 else [lambda *a: oracle.sgemmtr(*a, variant=0),
                                            lambda *a: oracle.sgemmtr(*a, variant=1)]
    want = np.array(case["expected"], dt)
    for fn in fns:
        C = np.array(case["C"], dt)
        for tA, tB, m, A, lda, B, ldb, beta in as_gemmtr_passes(case):
            C = run_gemmtr(fn, dt, case, tA, tB, m, A, lda, B, ldb, beta, C)
        assert bits_equal(C, want), (case["label"], C, want)


def test_gemmtr_golden_covers_the_reference_files():
    cases = load_golden("gemmtr_edge_cases.json")
    by = {}
    for c in cases:
        by[c["routine"]] = by.get(c["routine"], 0) + 1
    assert by == {"sgemmtr": 17, "dgemmtr": 17, "ssyrk": 14, "dsyrk": 14, "ssyr2k": 15, "dsyr2k": 15}
