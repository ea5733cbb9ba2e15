"""Generates the golden fixtures in tests/golden/ from the reference's own test data.

Run once in a checkout that has the reference tree (its path is the first
argument, default ../reference relative to the repo's parent); the outputs are
committed so the tests never read the reference at run time.

Outputs
-------
gemm_edge_cases.json
    Every case of the reference's tests/{sgemm,dgemm}/edge-cases.json and
    edge-cases-column-major.json (inputs copied as data), each with the exact
    expected C.
gemmtr_edge_cases.json
    The same for the gemmtr family, tests/{s,d}{gemmtr,syrk,syr2k}/edge-cases*.json:
    only the uplo triangle of C (col <= row for 'lower', col >= row for 'upper',
    in C's own terms) changes; syrk is gemmtr with B := A and the other
    transpose, syr2k two gemmtr passes, the second with beta = 1
    (src/ssyrk/ssyrk.mjs:29-31, src/ssyr2k/ssyr2k.mjs:25-26), each pass checked
    to be exact in f32.
symm_trmm_edge_cases.json
    The same for tests/{s,d}{symm,trmm}/edge-cases*.json: symm reads A's uplo
    triangle as a symmetric matrix (C := alpha*A*B + beta*C, or alpha*B*A + beta*C
    for side 'right'); trmm reads its uplo triangle, ones on the diagonal for
    diag 'unit', and overwrites B with alpha*op(A)*B (or alpha*B*op(A)). The reference checks these bit for bit against stdlib
    (tests/sgemm/src/test.sgemm.js:126-164,354-394; tests/dgemm/src/test.dgemm.js).
    Their values are small integers, so the expected output is computed here
    with exact rational arithmetic and then checked to be representable in f32:
    any correct GEMM must reproduce it exactly.
strsm_edge_cases.json
    The cases of tests/strsm/edge-cases*.json (inputs copied as data), each with
    X = op(A)^-1 * alpha*B solved in exact rational arithmetic and rounded to
    f32 ("expected"), and whether that solution is exact in f32 ("exact"). The
    reference checks strsm by its backward residual
    (tests/strsm/helpers.js, factor <= 5 in tests/strsm/src/test.strsm.js), not
    bit for bit; the exact solution pins the restated stdlib oracle.
gemv_edge_cases.json
    The cases of tests/{sgemv,dgemv}/edge-cases*.json (inputs copied as data),
    each with the exact y := alpha*op(A)*x + beta*y (strided gaps of y kept),
    computed with rationals and checked to be exact in the routine's type; the
    reference compares these outputs bit for bit (tests/sgemv/src/test.sgemv.js:116-153).
dd_lanes.json
    The lane cases of tests/shaders/src/test.dekker.js:98-138 (inputs and the
    expected result of twoSum, twoProdBit, ddAdd and ddMul per lane), restated
    with the same rules: exact results for the error-free transforms, hi+lo
    within 2^-40 of the f64 value for the double-double ops, and (value, 0) for
    a non-finite hi.
validation_params.json
    The parameter specs the reference's sgemm/dgemm validation tests load
    (tests/validation/params/{device,trans,layout,m,n,k,alpha,beta,A,B,C,ld,uplo,side,diag,
    lda,x,incx,y,incy}.json,
    read by tests/sgemm/src/test.sgemm.js:23-56 and tests/sgemmtr/src/test.sgemmtr.js), copied as data: the invalid
    values with their expected error substrings and the edge values that must
    not throw. tests/validation_runner.py replays them.
mulberry32.json
    The first draws of mulberry32 (src/random/random.mjs:4-12) for the seeds the
    reference's GEMM tests use, computed by a second, independent restatement of
    the JS integer arithmetic in pure Python (arbitrary-precision ints masked to
    32 bits). The C oracle and the product library are both checked against it.
"""
from __future__ import annotations

import json
import math
import os
import sys
from fractions import Fraction

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def f32(x: float) -> float:
    """Math.fround: round to nearest f32, overflowing to +-Infinity."""
    with np.errstate(over="ignore"):
        return float(np.float32(x))


def op_elem(M, ld, layout, trans, row, col):
    """op(M)[row, col] for a matrix stored in `layout` (tests/sgemm/helpers.js:8-11)."""
    sr, sc = (col, row) if trans == "transpose" else (row, col)
    return M[sc * ld + sr] if layout == "column-major" else M[sr * ld + sc]


def c_index(ldc, layout, row, col):
    return col * ldc + row if layout == "column-major" else row * ldc + col


def exact_gemm(case, uplo=None):
    layout = case.get("layout", "row-major")
    m, n, k = case["m"], case["n"], case["k"]
    alpha, beta = Fraction(case["alpha"]), Fraction(case["beta"])
    out = list(case["C"])
    for i in range(m):
        for j in range(n):
            if (uplo == "lower" and j > i) or (uplo == "upper" and j < i):
                continue
            acc = Fraction(0)
            for p in range(k):
                acc += Fraction(op_elem(case["A"], case["lda"], layout, case["transA"], i, p)) * \
                    Fraction(op_elem(case["B"], case["ldb"], layout, case["transB"], p, j))
            ci = c_index(case["ldc"], layout, i, j)
            val = alpha * acc + (beta * Fraction(case["C"][ci]) if beta != 0 else 0)
            fv = float(val)
            if Fraction(fv) != val or f32(fv) != fv:
                raise ValueError(f"{case['label']}: result {val} is not exact in f32")
            out[ci] = fv
    return out


def edge_cases(ref):
    cases = []
    for routine in ("sgemm", "dgemm"):
        for fname in ("edge-cases.json", "edge-cases-column-major.json"):
            with open(os.path.join(ref, "tests", routine, fname)) as fh:
                for tc in json.load(fh):
                    case = {k: tc[k] for k in ("label", "transA", "transB", "m", "n", "k", "alpha",
                                                "A", "lda", "B", "ldb", "beta", "C", "ldc")}
                    case["layout"] = tc.get("layout", "row-major")
                    case["routine"] = routine
                    case["source"] = f"tests/{routine}/{fname}"
                    case["expected"] = exact_gemm(case)
                    cases.append(case)
    return cases


def _flip(trans):
    return "no-transpose" if trans == "transpose" else "transpose"


def exact_tr(case):
    """Expected C of a gemmtr / syrk / syr2k case (see the module docstring)."""
    r = case["routine"][1:]
    g = dict(case)
    if r == "gemmtr":
        return exact_gemm(g, case["uplo"])
    g.update(m=case["n"], transA=case["trans"], transB=_flip(case["trans"]))
    if r == "syrk":
        g.update(B=case["A"], ldb=case["lda"])
        return exact_gemm(g, case["uplo"])
    first = exact_gemm(g, case["uplo"])
    g.update(A=case["B"], lda=case["ldb"], B=case["A"], ldb=case["lda"], beta=1, C=first)
    return exact_gemm(g, case["uplo"])


def gemmtr_edge_cases(ref):
    cases = []
    keys = {"gemmtr": ("label", "uplo", "transA", "transB", "m", "n", "k", "alpha", "A", "lda", "B", "ldb",
                       "beta", "C", "ldc"),
            "syrk": ("label", "uplo", "trans", "n", "k", "alpha", "A", "lda", "beta", "C", "ldc"),
            "syr2k": ("label", "uplo", "trans", "n", "k", "alpha", "A", "lda", "B", "ldb", "beta", "C", "ldc")}
    for routine in ("sgemmtr", "dgemmtr", "ssyrk", "dsyrk", "ssyr2k", "dsyr2k"):
        for fname in ("edge-cases.json", "edge-cases-column-major.json"):
            with open(os.path.join(ref, "tests", routine, fname)) as fh:
                for tc in json.load(fh):
                    case = {k: tc[k] for k in keys[routine[1:]]}
                    case["layout"] = tc.get("layout", "row-major")
                    case["routine"] = routine
                    case["source"] = f"tests/{routine}/{fname}"
                    case["expected"] = exact_tr(case)
                    cases.append(case)
    return cases


def _elem(M, ld, layout, r, c):
    return M[c * ld + r] if layout == "column-major" else M[r * ld + c]


def exact_special(case):
    """Expected result (C for symm, B for trmm) of a symm / trmm edge case."""
    layout = case.get("layout", "row-major")
    m, n, side, uplo = case["m"], case["n"], case["side"], case["uplo"]
    order = m if side == "left" else n
    lower = uplo == "lower"
    trmm = case["routine"].endswith("trmm")

    def a(i, j):  # the symmetric / triangular operand, op applied for trmm
        if trmm and case["transA"] == "transpose":
            i, j = j, i
        if trmm:
            if i == j:
                return Fraction(1) if case["diag"] == "unit" else Fraction(_elem(case["A"], case["lda"], layout, i, i))
            inside = i > j if lower else i < j
            return Fraction(_elem(case["A"], case["lda"], layout, i, j)) if inside else Fraction(0)
        stored = i >= j if lower else i <= j
        return Fraction(_elem(case["A"], case["lda"], layout, i, j) if stored else
                        _elem(case["A"], case["lda"], layout, j, i))

    def b(i, j):
        return Fraction(_elem(case["B"], case["ldb"], layout, i, j))

    alpha = Fraction(case["alpha"])
    out = list(case["B"] if trmm else case["C"])
    ld = case["ldb"] if trmm else case["ldc"]
    for i in range(m):
        for j in range(n):
            acc = sum((a(i, p) * b(p, j) for p in range(order)), Fraction(0)) if side == "left" else \
                sum((b(i, p) * a(p, j) for p in range(order)), Fraction(0))
            val = alpha * acc
            if not trmm and case["beta"] != 0:
                val += Fraction(case["beta"]) * Fraction(_elem(case["C"], ld, layout, i, j))
            fv = float(val)
            if Fraction(fv) != val or f32(fv) != fv:
                raise ValueError(f"{case['label']}: result {val} is not exact in f32")
            out[(j * ld + i) if layout == "column-major" else (i * ld + j)] = fv
    return out


def symm_trmm_edge_cases(ref):
    cases = []
    keys = {"symm": ("label", "side", "uplo", "m", "n", "alpha", "A", "lda", "B", "ldb", "beta", "C", "ldc"),
            "trmm": ("label", "side", "uplo", "transA", "diag", "m", "n", "alpha", "A", "lda", "B", "ldb")}
    for routine in ("ssymm", "dsymm", "strmm", "dtrmm"):
        for fname in ("edge-cases.json", "edge-cases-column-major.json"):
            with open(os.path.join(ref, "tests", routine, fname)) as fh:
                for tc in json.load(fh):
                    case = {k: tc[k] for k in keys[routine[1:]]}
                    case["layout"] = tc.get("layout", "row-major")
                    case["routine"] = routine
                    case["source"] = f"tests/{routine}/{fname}"
                    case["expected"] = exact_special(case)
                    cases.append(case)
    return cases


def exact_trsm(case):
    """X with op(A) X = alpha B (left) or X op(A) = alpha B (right), exact rationals,
    over a copy of B (padding kept); returns (values rounded to f32, all exact)."""
    layout = case.get("layout", "row-major")
    m, n, side = case["m"], case["n"], case["side"]
    order = m if side == "left" else n
    nt = case["transA"] == "no-transpose"
    lower = case["uplo"] == "lower"

    def op(i, j):  # op(A)(i, j), zero outside the stored triangle
        r, c = (i, j) if nt else (j, i)
        if r == c:
            return Fraction(1) if case["diag"] == "unit" else Fraction(_elem(case["A"], case["lda"], layout, r, r))
        inside = r > c if lower else r < c
        return Fraction(_elem(case["A"], case["lda"], layout, r, c)) if inside else Fraction(0)

    alpha = Fraction(case["alpha"])
    rhs = [[alpha * Fraction(_elem(case["B"], case["ldb"], layout, i, j)) for j in range(n)] for i in range(m)]
    X = [[None] * n for _ in range(m)]
    op_lower = nt == lower
    if side == "left":  # rows of X, in dependency order
        rows = range(order) if op_lower else range(order - 1, -1, -1)
        for i in rows:
            for j in range(n):
                acc = rhs[i][j] - sum((op(i, k) * X[k][j] for k in range(order) if k != i and X[k][j] is not None),
                                      Fraction(0))
                X[i][j] = acc / op(i, i)
    else:  # columns of X
        cols = range(order - 1, -1, -1) if op_lower else range(order)
        for j in cols:
            for i in range(m):
                acc = rhs[i][j] - sum((X[i][k] * op(k, j) for k in range(order) if k != j and X[i][k] is not None),
                                      Fraction(0))
                X[i][j] = acc / op(j, j)
    out = list(case["B"])
    exact = True
    for i in range(m):
        for j in range(n):
            fv = f32(float(X[i][j]))
            exact = exact and Fraction(fv) == X[i][j]
            out[(j * case["ldb"] + i) if layout == "column-major" else (i * case["ldb"] + j)] = fv
    return out, exact


def strsm_edge_cases(ref):
    keys = ("label", "side", "uplo", "transA", "diag", "m", "n", "alpha", "A", "lda", "B", "ldb")
    cases = []
    for fname in ("edge-cases.json", "edge-cases-column-major.json"):
        with open(os.path.join(ref, "tests", "strsm", fname)) as fh:
            for tc in json.load(fh):
                case = {k: tc[k] for k in keys}
                case["layout"] = tc.get("layout", "row-major")
                case["routine"] = "strsm"
                case["source"] = f"tests/strsm/{fname}"
                case["expected"], case["exact"] = exact_trsm(case)
                cases.append(case)
    return cases


def exact_gemv(case):
    layout = case.get("layout", "row-major")
    m, n = case["m"], case["n"]
    no_t = case["trans"] == "no-transpose"
    xlen, ylen = (n, m) if no_t else (m, n)

    def a(i, j):
        return Fraction(_elem(case["A"], case["lda"], layout, i, j))

    out = list(case["y"])
    for r in range(ylen):
        acc = sum((a(r, p) if no_t else a(p, r)) * Fraction(case["x"][p * case["incx"]]) for p in range(xlen))
        val = Fraction(case["alpha"]) * acc + Fraction(case["beta"]) * Fraction(case["y"][r * case["incy"]])
        fv = float(val)
        if Fraction(fv) != val or (case["routine"] == "sgemv" and f32(fv) != fv):
            raise ValueError(f"{case['label']}: result {val} is not exact")
        out[r * case["incy"]] = fv
    return out


def gemv_edge_cases(ref):
    keys = ("label", "trans", "m", "n", "alpha", "A", "lda", "x", "incx", "beta", "y", "incy")
    cases = []
    for routine in ("sgemv", "dgemv"):
        for fname in ("edge-cases.json", "edge-cases-column-major.json"):
            with open(os.path.join(ref, "tests", routine, fname)) as fh:
                for tc in json.load(fh):
                    case = {k: tc[k] for k in keys}
                    case["layout"] = tc.get("layout", "row-major")
                    case["routine"] = routine
                    case["source"] = f"tests/{routine}/{fname}"
                    case["expected"] = exact_gemv(case)
                    cases.append(case)
    return cases


# ---- double-double lane cases (tests/shaders/src/test.dekker.js:98-138) ----

def dd_lanes():
    inf = math.inf
    nan = math.nan
    raw = [
        ("finite", [1.5, -7.25, 1e10, 3], [3 * 2**-30, 0.1, -3.3e9, 1 / 3]),
        ("Inf next to finite", [1.5, inf, -7.25, -inf], [0.1, 1, 2**-29, 2]),
        ("NaN next to finite", [nan, 1.5, 3, nan], [1, 0.1, 2**-29, 2]),
        ("overflow next to finite", [3e38, 1.5, -3e38, 2], [3e38, 0.25, -3e38, 1e-3]),
    ]

    def low(h):
        return f32(h * 2**-26) if math.isfinite(h) else 0.0

    def exact(v):
        h = f32(v)
        return {"hi": h, "lo": (v - h) if math.isfinite(h) else 0.0}

    def dd(v):
        h = f32(v)
        if math.isfinite(h):
            return {"value": v, "rel": 2**-40}
        return {"hi": h, "lo": 0.0}

    out = []
    for label, a_hi, b_hi in raw:
        ah = [f32(x) for x in a_hi]
        bh = [f32(x) for x in b_hi]
        al = [low(x) for x in ah]
        bl = [low(x) for x in bh]
        lanes = []
        for l in range(4):
            a, b = ah[l], bh[l]
            av, bv = a + al[l], b + bl[l]
            lanes.append({
                "a_hi": a, "a_lo": al[l], "b_hi": b, "b_lo": bl[l],
                "twoSum": exact(a + b),
                "twoProdBit": exact(a * b),
                "ddAdd": dd(av + bv),
                "ddMul": dd(av * bv),
            })
        out.append({"label": label, "lanes": lanes})
    return out


# ---- mulberry32, second restatement ----

def mulberry32_draws(seed: int, count: int):
    a = seed & 0xFFFFFFFF
    out = []
    for _ in range(count):
        a = (a + 0x6D2B79F5) & 0xFFFFFFFF
        t = ((a ^ (a >> 15)) * (1 | a)) & 0xFFFFFFFF
        t = ((t + (((t ^ (t >> 7)) * (61 | t)) & 0xFFFFFFFF)) & 0xFFFFFFFF) ^ t
        out.append(((t ^ (t >> 14)) & 0xFFFFFFFF) / 4294967296.0)
    return out


def _dump(obj, name):
    def enc(v):
        if isinstance(v, float):
            if math.isnan(v):
                return "NaN"
            if math.isinf(v):
                return "Infinity" if v > 0 else "-Infinity"
        if isinstance(v, dict):
            return {k: enc(x) for k, x in v.items()}
        if isinstance(v, list):
            return [enc(x) for x in v]
        return v

    with open(os.path.join(HERE, name), "w") as fh:
        json.dump(enc(obj), fh, indent=1)
        fh.write("\n")


def validation_params(ref):
    names = ["device", "trans", "layout", "m", "n", "k", "alpha", "beta", "A", "B", "C", "ld", "uplo", "side", "diag",
             "lda", "x", "incx", "y", "incy"]
    out = {}
    for name in names:
        with open(os.path.join(ref, "tests", "validation", "params", f"{name}.json")) as fh:
            out[name] = json.load(fh)
    return out


def main():
    ref = sys.argv[1] if len(sys.argv) > 1 else os.path.join(HERE, "..", "..", "..", "reference")
    _dump(edge_cases(ref), "gemm_edge_cases.json")
    _dump(gemmtr_edge_cases(ref), "gemmtr_edge_cases.json")
    _dump(symm_trmm_edge_cases(ref), "symm_trmm_edge_cases.json")
    _dump(strsm_edge_cases(ref), "strsm_edge_cases.json")
    _dump(gemv_edge_cases(ref), "gemv_edge_cases.json")
    _dump(dd_lanes(), "dd_lanes.json")
    _dump(validation_params(ref), "validation_params.json")
    seeds = [0, 1, 2, 3, 42, 100, 111, 112, 113, 200, 300]
    _dump({"draws": 16, "seeds": {str(s): mulberry32_draws(s, 16) for s in seeds}}, "mulberry32.json")


if __name__ == "__main__":
    main()
