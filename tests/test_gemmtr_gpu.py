"""The gemmtr family on the GPU (sgemmtr/dgemmtr, ssyrk/dsyrk, ssyr2k/dsyr2k):
the reference's edge cases bit for bit, its validation specs, and random
products on every kernel path (FFMA/DFMA, 3xTF32 tensor cores, FP64 DMMA)
against the oracle. Only the uplo triangle may change; everything else in C,
including leading-dimension padding, must come back bit-identical."""
from __future__ import annotations

import numpy as np
import pytest

import validation_runner as vr
from conftest import bits_equal, load_golden
from test_gemmtr_oracle import as_gemmtr_passes, run_gemmtr

pytestmark = pytest.mark.gpu
ROUTINES = ("sgemmtr", "dgemmtr", "ssyrk", "dsyrk", "ssyr2k", "dsyr2k")


def call(wg, device, case, A, B, C):
    r, lay = case["routine"], case["layout"]
    fn = getattr(wg, r)
    if r.endswith("gemmtr"):
        return fn(device, case["uplo"], case["transA"], case["transB"], case["m"], case["n"], case["k"],
                  case["alpha"], A, case["lda"], B, case["ldb"], case["beta"], C, case["ldc"], lay)
    if r.endswith("syrk"):
        return fn(device, case["uplo"], case["trans"], case["n"], case["k"], case["alpha"], A, case["lda"],
                  case["beta"], C, case["ldc"], lay)
    return fn(device, case["uplo"], case["trans"], case["n"], case["k"], case["alpha"], A, case["lda"], B,
              case["ldb"], case["beta"], C, case["ldc"], lay)


@pytest.mark.parametrize("case", load_golden("gemmtr_edge_cases.json"),
                         ids=lambda c: f"{c['routine']}:{c['label'][:40]}")
def test_edge_cases_exact(wg, device, case):
    dt = np.float64 if case["routine"].startswith("d") else np.float32
    A = np.array(case["A"], dt)
    B = np.array(case["B"], dt) if "B" in case else None
    C = np.array(case["C"], dt)
    got = call(wg, device, case, A, B, C)["C"]
    assert bits_equal(got, np.array(case["expected"], dt)), (got, case["expected"])
    assert bits_equal(C, np.array(case["C"], dt)), "the input C was modified"


@pytest.mark.parametrize("routine", ROUTINES)
def test_validation_specs(wg, device, routine):
    fn = getattr(wg, routine)
    for label, args, err in vr.cases(routine, device, "invalid"):
        with pytest.raises(wg.Error) as ei:
            vr.call(fn, args)
        assert err in str(ei.value), label
    n = 0
    for label, args, _ in vr.cases(routine, device, "edge"):
        assert "C" in vr.call(fn, args), label
        n += 1
    assert n >= 10


def random_case(routine, uplo, layout, n, k, m=None, trans="no-transpose", transB="transpose", pad=3, seed=1,
                alpha=0.75, beta=-0.5):
    """A seeded case in the golden cases' format (stored operands with padded leading dimensions)."""
    rng = np.random.default_rng(seed)
    dt = np.float64 if routine.startswith("d") else np.float32
    cm = layout == "column-major"
    case = {"routine": routine, "uplo": uplo, "layout": layout, "n": n, "k": k, "alpha": alpha, "beta": beta}
    if routine.endswith("gemmtr"):
        ta, tb = trans, transB
        case.update(m=m, transA=ta, transB=tb)
        a_rows, a_cols = (m, k) if ta == "no-transpose" else (k, m)
        b_rows, b_cols = (k, n) if tb == "no-transpose" else (n, k)
    else:
        case.update(trans=trans)
        m = n
        a_rows, a_cols = (n, k) if trans == "no-transpose" else (k, n)
        b_rows, b_cols = a_rows, a_cols
    # stored: row-major rows x cols with ld >= cols, or column-major with ld >= rows
    lda = (a_rows if cm else a_cols) + pad
    ldb = (b_rows if cm else b_cols) + pad
    ldc = (m if cm else n) + pad
    case["A"] = (rng.random(lda * (a_cols if cm else a_rows)) * 2 - 1).astype(dt)
    case["B"] = (rng.random(ldb * (b_cols if cm else b_rows)) * 2 - 1).astype(dt)
    case["C"] = (rng.random(ldc * (n if cm else m)) * 2 - 1).astype(dt)
    case.update(lda=lda, ldb=ldb, ldc=ldc)
    return case


def oracle_result(oracle, case, fn):
    """The case through the oracle's gemmtr restatement `fn` (one or two passes)."""
    dt = case["C"].dtype
    C = case["C"].copy()
    for tA, tB, m, A, lda, B, ldb, beta in as_gemmtr_passes(case):
        C = run_gemmtr(fn, dt, case, tA, tB, m, A, lda, B, ldb, beta, C)
    return C


def triangle_mask(case):
    """True on the stored elements of C in the uplo triangle (C's own terms)."""
    m = case["m"] if case["routine"].endswith("gemmtr") else case["n"]
    n, ldc = case["n"], case["ldc"]
    i, j = np.meshgrid(np.arange(m), np.arange(n), indexing="ij")
    keep = (j <= i) if case["uplo"] == "lower" else (j >= i)
    idx = (j * ldc + i) if case["layout"] == "column-major" else (i * ldc + j)
    mask = np.zeros(case["C"].size, bool)
    mask[idx[keep]] = True
    return mask


def check_against(oracle, case, got, exact):
    f64 = case["routine"].startswith("d")
    mask = triangle_mask(case)
    assert bits_equal(got[~mask], case["C"][~mask]), "an element outside the triangle changed"
    if exact:
        fn = oracle.dgemmtr_fma if f64 else (lambda *a: oracle.sgemmtr(*a, variant=1))
        assert bits_equal(got, oracle_result(oracle, case, fn))
        return
    # fp64 truth of the same passes and a bound of the north-star form per pass
    fn64 = oracle.dgemmtr_fma
    c64 = dict(case, A=case["A"].astype(np.float64), B=case["B"].astype(np.float64), C=case["C"].astype(np.float64))
    truth = oracle_result(oracle, c64, fn64)
    absc = dict(c64, A=np.abs(c64["A"]), B=np.abs(c64["B"]), C=np.abs(c64["C"]), alpha=abs(case["alpha"]),
                beta=abs(case["beta"]))
    scale = oracle_result(oracle, absc, fn64)  # |alpha| sum|a||b| (+ the other pass) + |beta||c|
    eps = 2.0**-53 * 4 if f64 else 2.0**-24 * 2
    passes = len(as_gemmtr_passes(case))
    bound = passes * eps * max(case["k"], 1) * scale
    err = np.abs(got.astype(np.float64) - truth)
    assert np.all(err[mask] <= bound[mask]), float(np.max(err[mask] / np.where(bound[mask] > 0, bound[mask], 1)))


@pytest.mark.parametrize("routine", ROUTINES)
@pytest.mark.parametrize("uplo", ["lower", "upper"])
@pytest.mark.parametrize("layout", ["column-major", "row-major"])
@pytest.mark.parametrize("spath", ["simt", "simt_small"])
def test_simt_paths_bit_exact(wg, device, oracle, routine, uplo, layout, spath):
    """Small products run the FFMA / DFMA kernels: bit for bit the FMA restatement."""
    device.set_sgemm_path(spath)
    device.set_dgemm_path("simt")
    try:
        seed = ROUTINES.index(routine) * 4 + (uplo == "upper") * 2 + (layout == "row-major")
        case = random_case(routine, uplo, layout, n=70, k=33, m=90, seed=seed)
        got = call(wg, device, case, case["A"], case["B"], case["C"])["C"]
    finally:
        device.set_sgemm_path("auto")
        device.set_dgemm_path("auto")
    check_against(oracle, case, got, exact=True)


@pytest.mark.parametrize("routine", ROUTINES)
@pytest.mark.parametrize("uplo", ["lower", "upper"])
@pytest.mark.parametrize("trans", ["no-transpose", "transpose"])
def test_tensor_core_paths(wg, device, oracle, routine, uplo, trans):
    """Products large enough for the 3xTF32 / DMMA kernels: tiles outside the
    triangle are skipped, diagonal tiles masked, the rest within the bound."""
    before = device.sgemm_stats()
    case = random_case(routine, uplo, "column-major", n=600, k=300, m=700, trans=trans, seed=7)
    device.set_sgemm_path("tf32x3")  # auto sends a product this small to the FFMA kernel
    try:
        got = call(wg, device, case, case["A"], case["B"], case["C"])["C"]
    finally:
        device.set_sgemm_path("auto")
    if routine.startswith("s"):
        passes = len(as_gemmtr_passes(case))
        assert device.sgemm_stats()["tf32x3_launches"] - before["tf32x3_launches"] == passes
    check_against(oracle, case, got, exact=False)


def test_gpumatrix_in_place(wg, device, oracle):
    case = random_case("sgemmtr", "upper", "column-major", n=520, k=130, m=300, pad=0, seed=11)
    m, n, k = case["m"], case["n"], case["k"]
    GA = wg.GpuMatrix.from_(device, case["A"], m, k, case["lda"], "column-major")
    GB = wg.GpuMatrix.from_(device, case["B"], n, k, case["ldb"], "column-major")
    GC = wg.GpuMatrix.from_(device, case["C"], m, n, case["ldc"], "column-major")
    try:
        r = wg.sgemmtr(device, "upper", case["transA"], case["transB"], m, n, k, case["alpha"], GA,
                       case["lda"], GB, case["ldb"], case["beta"], GC, case["ldc"])
        assert "C" not in r  # GpuMatrix C is updated in place
        got = GC.read()
    finally:
        for g in (GA, GB, GC):
            g.destroy()
    check_against(oracle, case, got, exact=False)


def test_dgemmtr_quick_return_and_alpha_zero(wg, device):
    case = random_case("dgemmtr", "lower", "row-major", n=40, k=20, m=30, alpha=0.0, beta=1.0)
    got = call(wg, device, case, case["A"], case["B"], case["C"])["C"]
    assert bits_equal(got, case["C"])
    case = random_case("sgemmtr", "lower", "row-major", n=40, k=20, m=30, alpha=0.0, beta=2.0)
    got = call(wg, device, case, case["A"], case["B"], case["C"])["C"]
    mask = triangle_mask(case)
    assert bits_equal(got[mask], (np.float32(2.0) * case["C"][mask]).astype(np.float32))
    assert bits_equal(got[~mask], case["C"][~mask])


@pytest.mark.parametrize("path", ["tf32x3_packed", "tf32x3"])
@pytest.mark.parametrize("uplo", ["lower", "upper"])
@pytest.mark.parametrize("bad", [np.inf, np.nan])
def test_tensor_core_fallback_keeps_the_triangle(wg, device, oracle, path, uplo, bad):
    """A non-finite operand on the tensor-core paths: the split pass + MMA kernel
    computes the whole call's C on the FFMA pipe itself, the fused kernel ('tf32x3'
    at this size) the flagged tiles (the 128-row band holding the bad row of op(A)).
    Those come out bit for bit as the FMA restatement, the rest within the fp32
    bound, and nothing outside the triangle is touched."""
    case = random_case("sgemmtr", uplo, "column-major", n=520, k=200, m=600, pad=0, seed=29)
    case["A"][7 + 3 * case["lda"]] = bad  # op(A) row 7
    before = device.sgemm_stats()
    device.set_sgemm_path(path)
    try:
        got = call(wg, device, case, case["A"], case["B"], case["C"])["C"]
    finally:
        device.set_sgemm_path("auto")
    after = device.sgemm_stats()
    assert after["tf32x3_launches"] > before["tf32x3_launches"]
    assert after["fallbacks"] == before["fallbacks"] + 1
    mask = triangle_mask(case)
    assert bits_equal(got[~mask], case["C"][~mask]), "an element outside the triangle changed"
    want = oracle_result(oracle, case, lambda *a: oracle.sgemmtr(*a, variant=1))
    if path == "tf32x3_packed":
        assert bits_equal(got, want)
        return
    rows = np.arange(case["C"].size) % case["ldc"]
    band = mask & (rows < 128)
    assert bits_equal(got[band], want[band]), "the flagged tiles differ from the FMA restatement"
    rest = mask & (rows >= 128)
    c64 = dict(case, A=case["A"].astype(np.float64), B=case["B"].astype(np.float64), C=case["C"].astype(np.float64))
    truth = oracle_result(oracle, c64, oracle.dgemmtr_fma)
    absc = dict(c64, A=np.abs(c64["A"]), B=np.abs(c64["B"]), C=np.abs(c64["C"]), alpha=abs(case["alpha"]),
                beta=abs(case["beta"]))
    bound = 2.0**-24 * 2 * case["k"] * oracle_result(oracle, absc, oracle.dgemmtr_fma)
    assert np.all(np.abs(got[rest].astype(np.float64) - truth[rest]) <= bound[rest])
