"""sgemm on the GPU against the oracle: the reference's test cases
(tests/sgemm/src/test.sgemm.js and gpustorage.sgemm.js) plus the BASELINE configs."""
from __future__ import annotations

import math

import numpy as np
import pytest

import validation_runner as vr
from conftest import bits_equal, load_golden
from gemm_check import check_sgemm, fixture_args, ieee_match, sampled_columns_truth

pytestmark = pytest.mark.gpu
T, N = "transpose", "no-transpose"


def _call(wg, device, a, **kw):
    return wg.sgemm(device, a["transA"], a["transB"], a["m"], a["n"], a["k"], a["alpha"], a["A"], a["lda"],
                    a["B"], a["ldb"], a["beta"], a["C"], a["ldc"], a.get("layout", "row-major"), **kw)


def _check(oracle, got, a, exact=False):
    return check_sgemm(oracle, got, a["transA"], a["transB"], a["m"], a["n"], a["k"], a["alpha"], a["A"],
                       a["lda"], a["B"], a["ldb"], a["beta"], a["C"], a["ldc"], a.get("layout", "row-major"),
                       exact=exact)


@pytest.fixture(params=["simt", "simt_small"])
def simt(device, request):
    """Both FFMA kernels (128 x 128 and 32 x 64 tiles) run the same per-element
    arithmetic, so both match the FMA restatement bit for bit."""
    device.set_sgemm_path(request.param)
    yield device
    device.set_sgemm_path("auto")


# ---- test.sgemm.js:58-82 validation --------------------------------------------

def test_validation_invalid(wg, device):
    for label, args, err in vr.cases("sgemm", device, "invalid"):
        with pytest.raises(wg.Error) as ei:
            vr.call(wg.sgemm, args)
        assert err in str(ei.value), label


def test_validation_edge_cases_do_not_throw(wg, device):
    n = 0
    for label, args, _ in vr.cases("sgemm", device, "edge"):
        r = vr.call(wg.sgemm, args)
        assert "C" in r, label
        n += 1
    assert n >= 15


# ---- test.sgemm.js:93-122 fixtures: bit-exact against the FMA restatement -------------

def test_fixtures_bit_exact(wg, device, oracle, simt):
    rng = np.random.default_rng(0x5EED)
    for _ in range(100):
        a = fixture_args(rng, False)
        got = _call(wg, device, a)["C"]
        _check(oracle, got, a, exact=True)


def test_fixtures_gpumatrix(wg, device, oracle, simt):
    """gpustorage.sgemm.js:126-165: the same fixtures through resident GpuMatrix operands."""
    rng = np.random.default_rng(0x60B)
    for _ in range(30):
        a = fixture_args(rng, False)
        cm = a["layout"] == "column-major"
        a_rows, a_cols = (a["m"], a["k"]) if a["transA"] == N else (a["k"], a["m"])
        b_rows, b_cols = (a["k"], a["n"]) if a["transB"] == N else (a["n"], a["k"])
        GA = wg.GpuMatrix.from_(device, a["A"], a_rows, a_cols, a["lda"], a["layout"])
        GB = wg.GpuMatrix.from_(device, a["B"], b_rows, b_cols, a["ldb"], a["layout"])
        GC = wg.GpuMatrix.from_(device, a["C"], a["m"], a["n"], a["ldc"], a["layout"])
        try:
            r = wg.sgemm(device, a["transA"], a["transB"], a["m"], a["n"], a["k"], a["alpha"], GA, a["lda"],
                         GB, a["ldb"], a["beta"], GC, a["ldc"])
            assert set(r) == {"gpuTimeMs"} and r["gpuTimeMs"] >= 0
            dense = GC.read()
            ref = _call(wg, device, a)["C"]
            outer, inner = (a["n"], a["m"]) if cm else (a["m"], a["n"])
            want = np.concatenate([ref[o * a["ldc"]: o * a["ldc"] + inner] for o in range(outer)])
            assert bits_equal(dense, want)
        finally:
            for g in (GA, GB, GC):
                g.destroy()


# ---- test.sgemm.js:126-164, 354-394 edge cases: bit-exact ---------------------------

@pytest.mark.parametrize("case", [c for c in load_golden("gemm_edge_cases.json") if c["routine"] == "sgemm"],
                         ids=lambda c: c["label"][:50])
def test_edge_cases(wg, device, case):
    a = {k: case[k] for k in ("transA", "transB", "m", "n", "k", "alpha", "lda", "ldb", "beta", "ldc",
                              "layout")}
    for key in ("A", "B", "C"):
        a[key] = np.array(case[key], np.float32)
    got = _call(wg, device, a)["C"]
    assert bits_equal(got, np.array(case["expected"], np.float32))
    assert bits_equal(a["C"], np.array(case["C"], np.float32)), "input C was modified"


# ---- test.sgemm.js:175-230 large tile ---------------------------------------------

@pytest.mark.parametrize("ta", [N, T])
@pytest.mark.parametrize("tb", [N, T])
def test_large_tile_regression(wg, device, oracle, ta, tb):
    M = Nn = 400
    K = 8
    a_rows, a_cols = (M, K) if ta == N else (K, M)
    b_rows, b_cols = (K, Nn) if tb == N else (Nn, K)
    a = dict(transA=ta, transB=tb, m=M, n=Nn, k=K, alpha=1.5, A=wg.randomFloat32Array(a_rows * a_cols, -1, 1, 0),
             lda=a_cols, B=wg.randomFloat32Array(b_rows * b_cols, -1, 1, 100), ldb=b_cols, beta=0.5,
             C=wg.randomFloat32Array(M * Nn, -1, 1, 200), ldc=Nn)
    _check(oracle, _call(wg, device, a)["C"], a)


# ---- test.sgemm.js:239-296 ragged m, padded lda ------------------------------------

@pytest.mark.parametrize("mn", [(150, 70), (398, 390)])
@pytest.mark.parametrize("layout", ["row-major", "column-major"])
def test_ragged_padded(wg, device, oracle, mn, layout):
    M, Nn = mn
    K = 13
    cm = layout == "column-major"
    up4 = lambda v: (v + 3) // 4 * 4  # noqa: E731
    for ta in (N, T):
        for tb in (N, T):
            aR, aC = (M, K) if ta == N else (K, M)
            bR, bC = (K, Nn) if tb == N else (Nn, K)
            lda, ldb = up4(aR if cm else aC), up4(bR if cm else bC)
            a = dict(transA=ta, transB=tb, m=M, n=Nn, k=K, alpha=1.5,
                     A=wg.randomFloat32Array((aC if cm else aR) * lda, -1, 1, 111), lda=lda,
                     B=wg.randomFloat32Array((bC if cm else bR) * ldb, -1, 1, 112), ldb=ldb, beta=0.5,
                     C=wg.randomFloat32Array(M * Nn, -1, 1, 113), ldc=M if cm else Nn, layout=layout)
            _check(oracle, _call(wg, device, a)["C"], a)


# ---- test.sgemm.js:304-351 k = 0 ------------------------------------------------------

def test_k0_is_beta_c(wg, device):
    C = wg.randomFloat32Array(16, -5, 5, 300)
    got = wg.sgemm(device, N, T, 4, 4, 0, 1.5, np.zeros(3, np.float32), 1, np.zeros(3, np.float32), 1,
                   0.5, C, 4)["C"]
    assert bits_equal(got, (np.float32(0.5) * C).astype(np.float32))


# ---- test.sgemm.js:399-443 alpha = 0 ----------------------------------------------------

@pytest.mark.parametrize("n", [7, 400])
@pytest.mark.parametrize("beta", [0.0, 0.5])
def test_alpha0_reads_neither_a_nor_b(wg, device, oracle, n, beta):
    A = wg.randomFloat32Array(n * n, -1, 1, 1)
    A[1 * n + 2] = np.nan
    B = wg.randomFloat32Array(n * n, -1, 1, 2)
    B[2 * n + 3] = np.inf
    C = wg.randomFloat32Array(n * n, -1, 1, 3)
    if beta == 0:
        C[4 * n + 4] = np.nan
    got = wg.sgemm(device, N, N, n, n, n, 0.0, A, n, B, n, beta, C, n)["C"]
    want = oracle.sgemm(0, 0, n, n, n, 0.0, B, n, A, n, beta, C, n)  # row-major: C^T = B^T A^T
    ieee_match(got, want, 1e-4)
    assert not np.any(np.isnan(got))


# ---- IEEE specials with alpha != 0 (the dgemm test's cases, applied to sgemm) -------------

@pytest.mark.parametrize("path", ["auto", "simt", "simt_small"])
@pytest.mark.parametrize("n", [7, 150, 300])
def test_ieee_specials(wg, device, oracle, n, path):
    device.set_sgemm_path(path)
    try:
        A = wg.randomFloat32Array(n * n, -1, 1, 1)
        A[1 * n + 2] = np.inf
        B = wg.randomFloat32Array(n * n, -1, 1, 2)
        B[3 * n + 4] = np.nan
        C = wg.randomFloat32Array(n * n, -1, 1, 3)
        C[0], C[5] = np.nan, np.inf
        got = wg.sgemm(device, N, N, n, n, n, 1.5, A, n, B, n, 0.0, C, n)["C"]
        want = oracle.sgemm(0, 0, n, n, n, 1.5, B, n, A, n, 0.0, np.zeros(n * n, np.float32), n)
        ieee_match(got, want, 1e-4)
    finally:
        device.set_sgemm_path("auto")


# ---- BASELINE configs ------------------------------------------------------------------

def test_config1_512_cubed(wg, device, oracle):
    """512^3 column-major NN, alpha=1.5, beta=0.5, U[-1,1] seeded."""
    n = 512
    a = dict(transA=N, transB=N, m=n, n=n, k=n, alpha=1.5, A=wg.randomFloat32Array(n * n, -1, 1, 1), lda=n,
             B=wg.randomFloat32Array(n * n, -1, 1, 2), ldb=n, beta=0.5, C=wg.randomFloat32Array(n * n, -1, 1, 3),
             ldc=n, layout="column-major")
    for path in ("auto", "simt", "simt_small"):
        device.set_sgemm_path(path)
        try:
            _check(oracle, _call(wg, device, a)["C"], a, exact=path.startswith("simt"))
        finally:
            device.set_sgemm_path("auto")


@pytest.mark.parametrize("ta", [N, T])
def test_config4_ragged_padded(wg, device, oracle, ta):
    """M=1000 N=1023 K=777, lda=1024 ldb=800 ldc=1040, alpha=0.3 beta=-2 (the two
    legal transB=N combinations; transB=T is rejected, see test_validation)."""
    m, n, k = 1000, 1023, 777
    cols_a = k if ta == N else m
    a = dict(transA=ta, transB=N, m=m, n=n, k=k, alpha=0.3, A=wg.randomFloat32Array(1024 * cols_a, -1, 1, 41),
             lda=1024, B=wg.randomFloat32Array(800 * n, -1, 1, 42), ldb=800, beta=-2.0,
             C=wg.randomFloat32Array(1040 * n, -1, 1, 43), ldc=1040, layout="column-major")
    for path in ("auto", "simt", "simt_small"):
        device.set_sgemm_path(path)
        try:
            _check(oracle, _call(wg, device, a)["C"], a, exact=path.startswith("simt"))
        finally:
            device.set_sgemm_path("auto")


@pytest.mark.parametrize("tb", [N, T])
def test_config4_added_nt_tt_with_legal_ldb(wg, device, oracle, tb):
    """Addition to configs[3]: NT / TT with the nearest legal ldb (1024)."""
    m, n, k = 1000, 1023, 777
    a = dict(transA=T, transB=tb, m=m, n=n, k=k, alpha=0.3, A=wg.randomFloat32Array(1024 * m, -1, 1, 51),
             lda=1024, B=wg.randomFloat32Array(1024 * (k if tb == T else n), -1, 1, 52), ldb=1024, beta=-2.0,
             C=wg.randomFloat32Array(1040 * n, -1, 1, 53), ldc=1040, layout="column-major")
    _check(oracle, _call(wg, device, a)["C"], a)


def test_config2_4096_full_size_sampled(wg, device, oracle):
    """configs[1] at full size: 4096^3 column-major TN, alpha=1, beta=0, A and B ~ N(0,1)
    seeded, C = 0. The whole result is computed on the GPU; 48 columns are checked
    against the fp64 truth (a full CPU product would take minutes)."""
    n = 4096
    A = wg.randomNormalFloat32Array(n * n, 11)
    B = wg.randomNormalFloat32Array(n * n, 12)
    C = np.zeros(n * n, np.float32)
    got = wg.sgemm(device, T, N, n, n, n, 1.0, A, n, B, n, 0.0, C, n, "column-major")["C"]
    cols = np.linspace(0, n - 1, 48).astype(int)
    truth, absab, Cs = sampled_columns_truth(oracle, False, 1, 0, n, n, n, 1.0, A, n, B, n, 0.0, C, n, cols)
    g = np.stack([got[j * n:(j + 1) * n] for j in cols], axis=1).astype(np.float64)
    t = oracle.dense(truth, n, len(cols))
    bound = oracle.sgemm_bound(n, len(cols), n, 1.0, absab, 0.0, Cs, n)
    assert np.all(np.abs(g - t) <= bound)
    assert np.all(np.isfinite(got))


def test_gpu_time_reported_on_benchmark_device(wg, device):
    a = np.ones(64 * 64, np.float32)
    r = wg.sgemm(device, N, N, 64, 64, 64, 1.0, a, 64, a, 64, 0.0, a, 64)
    assert r["gpuTimeMs"] > 0 and np.all(r["C"] == 64)
