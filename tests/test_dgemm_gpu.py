"""dgemm on the GPU against the oracle: the reference's test cases
(tests/dgemm/src/test.dgemm.js and gpustorage.dgemm.js) plus the BASELINE configs.

The reference computes dgemm in double-double with f32's exponent range; this
build uses native FP64, so results are held to the fp64 truth within
4*K*2^-53*(|alpha||A||B| + |beta||C|), and the one intended divergence — the
reference's f32 exponent range (tests/dgemm/src/test.dgemm.js:454-535) — is
checked to follow real f64 instead."""
from __future__ import annotations

import math

import numpy as np
import pytest

import validation_runner as vr
from conftest import bits_equal, load_golden
from gemm_check import check_dgemm, fixture_args, ieee_match, sampled_columns_truth

pytestmark = pytest.mark.gpu
T, N = "transpose", "no-transpose"


def _call(wg, device, a):
    return wg.dgemm(device, a["transA"], a["transB"], a["m"], a["n"], a["k"], a["alpha"], a["A"], a["lda"],
                    a["B"], a["ldb"], a["beta"], a["C"], a["ldc"], a.get("layout", "row-major"))


def _check(oracle, got, a, exact=False):
    return check_dgemm(oracle, got, a["transA"], a["transB"], a["m"], a["n"], a["k"], a["alpha"], a["A"],
                       a["lda"], a["B"], a["ldb"], a["beta"], a["C"], a["ldc"], a.get("layout", "row-major"),
                       exact=exact)


def test_validation_invalid(wg, device):
    def wrong_dtype():
        return wg.GpuMatrix.from_(device, np.ones(4, np.float32), 2, 2)

    for label, args, err in vr.cases("dgemm", device, "invalid", wrong_dtype):
        with pytest.raises(wg.Error) as ei:
            vr.call(wg.dgemm, args)
        assert err in str(ei.value), label


def test_validation_edge_cases_do_not_throw(wg, device):
    for label, args, _ in vr.cases("dgemm", device, "edge"):
        assert "C" in vr.call(wg.dgemm, args), label


def test_fixtures(wg, device, oracle):
    """test.dgemm.js fixtures: 100 random cases; bit-identical to the fp64 FMA
    restatement (the DFMA kernel's arithmetic) and within the fp64 bound."""
    rng = np.random.default_rng(0xD6E)
    worst_dd = 0.0
    for _ in range(100):
        a = fixture_args(rng, True)
        rep = _check(oracle, _call(wg, device, a)["C"], a, exact=True)
        worst_dd = max(worst_dd, rep["reference_dd_max_abs_err"])
    print(f"reference double-double max abs deviation from fp64 truth over fixtures: {worst_dd:.3e}")


def test_fixtures_gpumatrix(wg, device, oracle):
    rng = np.random.default_rng(0xD60)
    for _ in range(20):
        a = fixture_args(rng, True)
        cm = a["layout"] == "column-major"
        a_rows, a_cols = (a["m"], a["k"]) if a["transA"] == N else (a["k"], a["m"])
        b_rows, b_cols = (a["k"], a["n"]) if a["transB"] == N else (a["n"], a["k"])
        GA = wg.GpuMatrix.from_(device, a["A"], a_rows, a_cols, a["lda"], a["layout"])
        GB = wg.GpuMatrix.from_(device, a["B"], b_rows, b_cols, a["ldb"], a["layout"])
        GC = wg.GpuMatrix.from_(device, a["C"], a["m"], a["n"], a["ldc"], a["layout"])
        try:
            wg.dgemm(device, a["transA"], a["transB"], a["m"], a["n"], a["k"], a["alpha"], GA, a["lda"], GB,
                     a["ldb"], a["beta"], GC, a["ldc"])
            ref = _call(wg, device, a)["C"]
            outer, inner = (a["n"], a["m"]) if cm else (a["m"], a["n"])
            want = np.concatenate([ref[o * a["ldc"]: o * a["ldc"] + inner] for o in range(outer)])
            assert bits_equal(GC.read(), want)
        finally:
            for g in (GA, GB, GC):
                g.destroy()


@pytest.mark.parametrize("case", [c for c in load_golden("gemm_edge_cases.json") if c["routine"] == "dgemm"],
                         ids=lambda c: c["label"][:50])
def test_edge_cases(wg, device, case):
    a = {k: case[k] for k in ("transA", "transB", "m", "n", "k", "alpha", "lda", "ldb", "beta", "ldc",
                              "layout")}
    for key in ("A", "B", "C"):
        a[key] = np.array(case[key], np.float64)
    assert bits_equal(_call(wg, device, a)["C"], np.array(case["expected"], np.float64))


def _full_precision(n, seed):
    """Doubles that need all 53 bits (tests/helpers/exactness.js: fullPrecisionFrom)."""
    return wg_random(n, seed) + 1 / 3


def wg_random(n, seed):
    import wgblas_b200

    return wgblas_b200.randomFloat64Array(n, -1, 1, seed)


@pytest.mark.parametrize("alpha,k", [(0.0, 6), (1.5, 0)])
def test_exactness_quick_return(wg, device, alpha, k):
    """test.dgemm.js:353-381: alpha=0 or k=0 with beta=1 returns C itself, bit-identical."""
    n = 6
    A = np.zeros(n, np.float64) if k == 0 else _full_precision(n * k, 1030)
    B = np.zeros(1, np.float64) if k == 0 else _full_precision(k * n, 1031)
    C = _full_precision(n * n, 1032)
    want = C.copy()
    got = wg.dgemm(device, N, N, n, n, k, alpha, A, max(k, 1), B, n, 1.0, C, n)["C"]
    assert got is C and bits_equal(got, want)


def test_exactness_ldc_padding(wg, device):
    """test.dgemm.js:382-407: the ldc gap comes back bit-identical."""
    n, m, k, ldc = 6, 4, 2, 9
    C = _full_precision(m * ldc, 1040)
    got = wg.dgemm(device, N, N, m, n, k, 1.5, _full_precision(m * k, 1041), k, _full_precision(k * n, 1042),
                   n, 0.5, C, ldc)["C"]
    pad = np.ones(C.size, bool)
    for i in range(m):
        pad[i * ldc: i * ldc + n] = False
    assert bits_equal(got[pad], C[pad])


@pytest.mark.parametrize("n", [7, 150])
def test_ieee_specials(wg, device, oracle, n):
    """test.dgemm.js:410-452: Inf in A, NaN in B; beta=0 ignores NaN/Inf in C."""
    A = wg_random(n * n, 1)
    A[1 * n + 2] = np.inf
    B = wg_random(n * n, 2)
    B[3 * n + 4] = np.nan
    C = wg_random(n * n, 3)
    C[0], C[5] = np.nan, np.inf
    got = wg.dgemm(device, N, N, n, n, n, 1.5, A, n, B, n, 0.0, C, n)["C"]
    truth, _ = oracle.dgemm_truth(0, 0, n, n, n, 1.5, B, n, A, n, 0.0, np.zeros(n * n), n)
    ieee_match(got, truth, 1e-12)


@pytest.mark.parametrize("n", [7, 150])
def test_f64_exponent_range_follows_real_f64(wg, device, oracle, n):
    """The intended divergence from test.dgemm.js:454-535: values beyond f32's range
    (1e300, 1e-50) are kept as real f64 does, not saturated as double-double does."""
    A = wg_random(n * n, 1)
    A[4 * n + 2], A[5 * n + 5] = 1e300, 1e-50
    B = wg_random(n * n, 2)
    B[5 * n + 1] = -1e-50
    C = wg_random(n * n, 3)
    C[6 * n + 6] = -1e300
    got = wg.dgemm(device, N, N, n, n, n, 1.5, A, n, B, n, 0.5, C, n)["C"]
    truth, _ = oracle.dgemm_truth(0, 0, n, n, n, 1.5, B, n, A, n, 0.5, C, n)
    ieee_match(got, truth, 1e-9)
    assert np.all(np.isfinite(got))
    dd = oracle.dgemm_dd(0, 0, n, n, n, 1.5, B, n, A, n, 0.5, C, n)
    assert not np.all(np.isfinite(dd)), "the double-double restatement saturates, as the reference does"


@pytest.mark.parametrize("n", [7, 150])
@pytest.mark.parametrize("beta", [0.0, 0.5])
def test_alpha0_reads_neither_a_nor_b(wg, device, oracle, n, beta):
    A = wg_random(n * n, 1)
    A[1 * n + 2] = np.nan
    B = wg_random(n * n, 2)
    B[2 * n + 3] = np.inf
    C = wg_random(n * n, 3)
    if beta == 0:
        C[4 * n + 4] = np.nan
    got = wg.dgemm(device, N, N, n, n, n, 0.0, A, n, B, n, beta, C, n)["C"]
    want = oracle.dgemm_fma(0, 0, n, n, n, 0.0, B, n, A, n, beta, C, n)
    ieee_match(got, want, 1e-9)


def test_config3_4096_full_size_sampled(wg, device, oracle):
    """configs[2] at full size: 4096^3 column-major NT, alpha=-0.75, beta=1.25, U[-1,1]
    seeded; 48 columns checked against the long-double truth, and the reference's
    double-double deviation on the same columns reported."""
    n = 4096
    A = wg_random(n * n, 21)
    B = wg_random(n * n, 22)
    C = wg_random(n * n, 23)
    got = wg.dgemm(device, N, T, n, n, n, -0.75, A, n, B, n, 1.25, C, n, "column-major")["C"]
    cols = np.linspace(0, n - 1, 48).astype(int)
    truth, absab, Cs = sampled_columns_truth(oracle, True, 0, 1, n, n, n, -0.75, A, n, B, n, 1.25, C, n, cols)
    g = np.stack([got[j * n:(j + 1) * n] for j in cols], axis=1)
    t = oracle.dense(truth, n, len(cols))
    bound = oracle.dgemm_bound(n, len(cols), n, -0.75, absab, 1.25, Cs, n)
    assert np.all(np.abs(g - t) <= bound)


# ---- the FP64 tensor-core (DMMA) kernel, forced on ------------------------------------

@pytest.fixture
def dmma(device):
    device.set_dgemm_path("dmma")
    yield device
    device.set_dgemm_path("auto")


@pytest.mark.parametrize("shape", [(128, 128, 16), (200, 300, 77), (512, 512, 512), (1000, 1023, 777),
                                   (129, 257, 40), (7, 9, 3)])
@pytest.mark.parametrize("ta", [N, T])
@pytest.mark.parametrize("tb", [N, T])
def test_dmma_shapes_and_transposes(wg, device, oracle, dmma, shape, ta, tb):
    m, n, k = shape
    a_rows, a_cols = (m, k) if ta == N else (k, m)
    b_rows, b_cols = (k, n) if tb == N else (n, k)
    lda, ldb, ldc = a_rows + 3, b_rows + 1, m + 2
    a = dict(transA=ta, transB=tb, m=m, n=n, k=k, alpha=-0.75, A=wg_random(lda * a_cols, 61), lda=lda,
             B=wg_random(ldb * b_cols, 62), ldb=ldb, beta=1.25, C=wg_random(ldc * n, 63), ldc=ldc,
             layout="column-major")
    _check(oracle, _call(wg, device, a)["C"], a)


@pytest.mark.parametrize("n", [7, 150])
def test_dmma_ieee_specials(wg, device, oracle, dmma, n):
    test_ieee_specials(wg, device, oracle, n)


def test_dmma_same_sign_long_k(wg, device, oracle, dmma):
    m = n = 192
    k = 4096
    A = wgblas_uniform(m * k, 0.0, 1.0, 71)
    B = wgblas_uniform(k * n, 0.0, 1.0, 72)
    C = wgblas_uniform(m * n, 0.0, 1.0, 73)
    a = dict(transA=N, transB=N, m=m, n=n, k=k, alpha=1.0, A=A, lda=m, B=B, ldb=k, beta=1.0, C=C, ldc=m,
             layout="column-major")
    _check(oracle, _call(wg, device, a)["C"], a)


def wgblas_uniform(n, low, high, seed):
    import wgblas_b200

    return wgblas_b200.randomFloat64Array(n, low, high, seed)
