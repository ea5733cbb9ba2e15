"""Pins the CPU oracle (oracle/) to the reference's own known answers. CPU only.

* edge cases: tests/{sgemm,dgemm}/edge-cases*.json with their exact results
  (tests/golden/gemm_edge_cases.json), bit for bit, for every restatement;
* double-double primitives: the lane cases of tests/shaders/src/test.dekker.js;
* split / merge: the cases of tests/utils/test.f64.js;
* mulberry32: a second restatement of src/random/random.mjs:4-12;
* the forward-error bounds of tests/sgemm/helpers.js and tests/dgemm/helpers.js
  on seeded fixtures like the reference's (tests/helpers/fixtures.js).
"""
from __future__ import annotations

import math

import numpy as np
import pytest

from conftest import bits_equal, load_golden


def _frame(case):
    """Column-major-frame arguments for a golden case (layout per the case)."""
    cm = case["layout"] == "column-major"
    ta = (case["transA"] == "transpose") == cm
    tb = (case["transB"] == "transpose") == cm
    if cm:
        return int(ta), int(tb), case["m"], case["n"], "A", case["lda"], "B", case["ldb"]
    return int(not tb), int(not ta), case["n"], case["m"], "B", case["ldb"], "A", case["lda"]


@pytest.mark.parametrize("case", load_golden("gemm_edge_cases.json"), ids=lambda c: f"{c['routine']}:{c['label'][:40]}")
def test_edge_cases_exact(oracle, case):
    ta, tb, m, n, an, lda, bn, ldb = _frame(case)
    k = case["k"]
    if case["routine"] == "sgemm":
        A = np.array(case[an], np.float32)
        B = np.array(case[bn], np.float32)
        C = np.array(case["C"], np.float32)
        want = np.array(case["expected"], np.float32)
        for variant in (0, 1):
            got = oracle.sgemm(ta, tb, m, n, k, case["alpha"], A, lda, B, ldb, case["beta"], C, case["ldc"],
                               variant=variant)
            assert bits_equal(got, want), (variant, got, want)
    else:
        A = np.array(case[an], np.float64)
        B = np.array(case[bn], np.float64)
        C = np.array(case["C"], np.float64)
        want = np.array(case["expected"], np.float64)
        for fn in (lambda *a: oracle.dgemm_dd(*a, variant=0), lambda *a: oracle.dgemm_dd(*a, variant=1),
                   oracle.dgemm_fma):
            got = fn(ta, tb, m, n, k, case["alpha"], A, lda, B, ldb, case["beta"], C, case["ldc"])
            assert bits_equal(got, want), (got, want)


# ---- double-double lanes: tests/shaders/src/test.dekker.js:98-155 ----

def _check_dd(got, want, where):
    hi, lo = float(got[0]), float(got[1])
    if "value" in want:
        v = hi + lo
        err = abs(v - want["value"]) / abs(want["value"])
        assert err <= want["rel"], f"{where}: hi+lo={v} want {want['value']} (rel {err})"
        return
    if math.isnan(want["hi"]):
        assert math.isnan(hi), where
    else:
        assert hi == want["hi"] and math.copysign(1, hi) == math.copysign(1, want["hi"]), where
    if math.isfinite(want["hi"]):
        assert lo == want["lo"], f"{where}: lo={lo} want {want['lo']}"
    else:
        assert lo == 0, f"{where}: non-finite hi must carry a zero error term, got {lo}"


@pytest.mark.parametrize("group", load_golden("dd_lanes.json"), ids=lambda g: g["label"])
def test_dd_lanes(oracle, group):
    for i, ln in enumerate(group["lanes"]):
        where = f"{group['label']} lane {i}"
        _check_dd(oracle.dd_two_sum(ln["a_hi"], ln["b_hi"]), ln["twoSum"], where + " twoSum")
        _check_dd(oracle.dd_two_prod_bit(ln["a_hi"], ln["b_hi"]), ln["twoProdBit"], where + " twoProdBit")
        _check_dd(oracle.dd_add(ln["a_hi"], ln["a_lo"], ln["b_hi"], ln["b_lo"]), ln["ddAdd"], where + " ddAdd")
        _check_dd(oracle.dd_mul(ln["a_hi"], ln["a_lo"], ln["b_hi"], ln["b_lo"]), ln["ddMul"], where + " ddMul")


# ---- split / merge: tests/utils/test.f64.js ----

def test_split_is_round_and_residual(oracle):
    x = np.array([math.pi, math.e, 1 / 3])
    hi, lo = oracle.dd_split(x)
    assert np.array_equal(hi, x.astype(np.float32))
    assert np.array_equal(lo, (x - hi.astype(np.float64)).astype(np.float32))


def test_round_trip_beats_f32(oracle):
    x = np.array([math.pi, math.e, 1 / 3, 0.1, 1e-7, 123456.789, -math.pi, -1e-30, 1e-30, -0.1])
    hi, lo = oracle.dd_split(x)
    merged = oracle.dd_merge(hi, lo)
    assert np.all(np.abs(merged - x) <= np.abs(x.astype(np.float32).astype(np.float64) - x))
    assert np.all(np.abs(merged - x) / np.abs(x) < 2.0**-40)
    assert np.all(np.sign(merged) == np.sign(x))


def test_exact_f32_values_have_zero_lo(oracle):
    x = np.array([0, 0.5, 2, -8, 1024], np.float64)
    hi, lo = oracle.dd_split(x)
    assert np.all(lo == 0) and np.array_equal(oracle.dd_merge(hi, lo), x)


def test_merge_is_elementwise_sum(oracle):
    got = oracle.dd_merge(np.array([1, 2, -3], np.float32), np.array([0.5, -0.25, 0.125], np.float32))
    assert list(got) == [1.5, 1.75, -2.875]


def test_merge_exact_restores_unchanged(oracle):
    before = np.array([1 / 3, math.pi, 2.5, -0.0, math.inf])
    hi, lo = oracle.dd_split(before)
    assert oracle.dd_merge(hi, lo)[0] != before[0]
    hi[2], lo[2] = 7, 0
    out = oracle.dd_merge_exact(hi, lo, before)
    assert out[0] == 1 / 3 and out[1] == math.pi and out[2] == 7
    assert out[3] == 0 and math.copysign(1, out[3]) == -1 and out[4] == math.inf


def test_merge_exact_merges_changed(oracle):
    before = np.array([1 / 3])
    hi, lo = oracle.dd_split(before)
    lo[0] = np.float32(lo[0] * 2)
    out = oracle.dd_merge_exact(hi, lo, before)
    assert out[0] == float(hi[0]) + float(lo[0]) and out[0] != before[0]


def test_split_specials(oracle):
    hi, lo = oracle.dd_split(np.array([math.inf, -math.inf, math.nan]))
    assert hi[0] == math.inf and hi[1] == -math.inf and math.isnan(hi[2])
    assert np.all(lo == 0)


def test_merge_exact_never_restores_out_of_range(oracle):
    before = np.array([1e300, 1e-320, math.inf])
    hi, lo = oracle.dd_split(before)
    out = oracle.dd_merge_exact(hi, lo, before)
    assert out[0] == math.inf and out[1] == 0 and out[2] == math.inf


# ---- mulberry32 ----

def test_mulberry32_matches_second_restatement(oracle):
    g = load_golden("mulberry32.json")
    for seed, draws in g["seeds"].items():
        got = oracle.random_f64(g["draws"], 0.0, 1.0, int(seed))
        assert list(got) == draws, seed


def test_random_f32_rounds_the_double_sum(oracle):
    g = load_golden("mulberry32.json")
    for seed, draws in g["seeds"].items():
        u = np.array(draws)
        want = (-3.0 + u * (5.0 - -3.0)).astype(np.float32)
        assert bits_equal(oracle.random_f32(len(draws), -3.0, 5.0, int(seed)), want)


def test_normal_is_standard(oracle):
    z = oracle.normal_f64(200000, 7).astype(np.float64)
    assert abs(z.mean()) < 0.01 and abs(z.std() - 1) < 0.01
    assert bits_equal(oracle.normal_f32(1001, 7), oracle.normal_f64(1001, 7).astype(np.float32))


# ---- forward-error bounds on seeded fixtures ----

def _fixture(rng, f64):
    m, n, k = (int(x) for x in rng.integers(1, 21, 3))
    ta, tb = (int(x) for x in rng.integers(0, 2, 2))
    lda = (k if ta else m) + int(rng.integers(0, 3))
    ldb = (n if tb else k) + int(rng.integers(0, 3))
    ldc = m + int(rng.integers(0, 3))

    def scalar():
        v = float(rng.uniform(-10, 10))
        return 0.0 if abs(v) < 1e-3 else v

    dt = np.float64 if f64 else np.float32
    A = rng.uniform(-10, 10, lda * (m if ta else k)).astype(dt)
    B = rng.uniform(-10, 10, ldb * (k if tb else n)).astype(dt)
    C = rng.uniform(-10, 10, ldc * n).astype(dt)
    return ta, tb, m, n, k, scalar(), A, lda, B, ldb, scalar(), C, ldc


def test_sgemm_restatement_within_reference_bound(oracle):
    rng = np.random.default_rng(20240601)
    for _ in range(100):
        ta, tb, m, n, k, al, A, lda, B, ldb, be, C, ldc = _fixture(rng, False)
        al, be = float(np.float32(al)), float(np.float32(be))
        truth, absab = oracle.sgemm_truth(ta, tb, m, n, k, al, A, lda, B, ldb, be, C, ldc)
        for variant in (0, 1):
            got = oracle.sgemm(ta, tb, m, n, k, al, A, lda, B, ldb, be, C, ldc, variant=variant)
            ff = oracle.forward_factor(got, truth, m, n, k, al, absab, be, C, ldc, 2.0**-23, 1, 1)
            assert ff <= 1, (variant, ff)


def test_dgemm_restatements_within_reference_bound(oracle):
    """The double-double restatement stays near the reference's own bound
    (tests/dgemm/helpers.js: eps=2^-48, (k+2)|alpha|, 3|beta|). That bound is not
    a guarantee of the algorithm: on rare wide-double inputs (k=1, |alpha|~5) the
    restated arithmetic reaches 1.08x it unfused and 1.22x with the cross terms
    fused, so the reference's deviation is measured and reported, and held here
    below 1.5x. The native fp64 restatement must meet the north-star bound
    4*K*2^-53*(|alpha||A||B| + |beta||C|) outright."""
    rng = np.random.default_rng(20240602)
    worst = 0.0
    for _ in range(100):
        ta, tb, m, n, k, al, A, lda, B, ldb, be, C, ldc = _fixture(rng, True)
        truth, absab = oracle.dgemm_truth(ta, tb, m, n, k, al, A, lda, B, ldb, be, C, ldc)
        for variant in (0, 1):
            dd = oracle.dgemm_dd(ta, tb, m, n, k, al, A, lda, B, ldb, be, C, ldc, variant=variant)
            worst = max(worst, oracle.forward_factor(dd, truth, m, n, k, al, absab, be, C, ldc,
                                                     2.0**-48, 2, 3))
        fm = oracle.dgemm_fma(ta, tb, m, n, k, al, A, lda, B, ldb, be, C, ldc)
        err = np.abs(oracle.block(fm, m, n, ldc) - oracle.dense(truth, m, n))
        assert np.all(err <= oracle.dgemm_bound(m, n, k, al, absab, be, C, ldc))
    assert worst < 1.5, worst


def test_sgemm_k0_is_beta_c(oracle):
    C = oracle.random_f32(16, -5, 5, 300)
    got = oracle.sgemm(0, 1, 4, 4, 0, 1.5, np.zeros(3, np.float32), 1, np.zeros(3, np.float32), 1, 0.5, C, 4)
    assert bits_equal(got, (np.float32(0.5) * C).astype(np.float32))


def test_dgemm_dd_quick_return_and_padding(oracle):
    rng = np.random.default_rng(5)
    C = rng.standard_normal(36)
    A = rng.standard_normal(36)
    assert bits_equal(oracle.dgemm_dd(0, 0, 6, 6, 6, 0.0, A, 6, A, 6, 1.0, C, 6), C)
    assert bits_equal(oracle.dgemm_dd(0, 0, 6, 6, 0, 1.5, A, 6, A, 6, 1.0, C, 6), C)
    # ldc padding is restored exactly by the exact merge
    Cp = rng.standard_normal(9 * 6)
    got = oracle.dgemm_dd(0, 0, 4, 6, 2, 1.5, A, 4, A, 2, 0.5, Cp, 9)
    pad = np.ones(9 * 6, bool)
    for j in range(6):
        pad[j * 9: j * 9 + 4] = False
    assert bits_equal(got[pad], Cp[pad])
