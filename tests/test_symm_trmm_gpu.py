"""ssymm/dsymm and strmm/dtrmm on the GPU: the reference's edge cases bit for
bit, its validation specs, and random products on the FFMA/DFMA kernels (bit
for bit against the oracle's restatement) and on the tensor-core kernels
(within the north-star bound of an fp64 truth). Everything outside the m x n
result block (leading-dimension padding) must come back unchanged."""
from __future__ import annotations

import numpy as np
import pytest

import validation_runner as vr
from conftest import bits_equal, load_golden
from test_symm_trmm_oracle import dense_operand, general, restate

pytestmark = pytest.mark.gpu
ROUTINES = ("ssymm", "dsymm", "strmm", "dtrmm")


def call(wg, device, case, A, B, C):
    fn = getattr(wg, case["routine"])
    if case["routine"].endswith("trmm"):
        return fn(device, case["side"], case["uplo"], case["transA"], case["diag"], case["m"], case["n"],
                  case["alpha"], A, case["lda"], B, case["ldb"], case["layout"])
    return fn(device, case["side"], case["uplo"], case["m"], case["n"], case["alpha"], A, case["lda"], B, case["ldb"],
              case["beta"], C, case["ldc"], case["layout"])


def result_key(case):
    return "B" if case["routine"].endswith("trmm") else "C"


@pytest.mark.parametrize("case", load_golden("symm_trmm_edge_cases.json"),
                         ids=lambda c: f"{c['routine']}:{c['label'][:40]}")
def test_edge_cases_exact(wg, device, case):
    dt = np.float64 if case["routine"].startswith("d") else np.float32
    A = np.array(case["A"], dt)
    B = np.array(case["B"], dt)
    C = np.array(case["C"], dt) if "C" in case else None
    got = call(wg, device, case, A, B, C)[result_key(case)]
    assert bits_equal(got, np.array(case["expected"], dt)), (got, case["expected"])
    assert bits_equal(B, np.array(case["B"], dt)), "the input B was modified"


@pytest.mark.parametrize("routine", ROUTINES)
def test_validation_specs(wg, device, routine):
    fn = getattr(wg, routine)
    for label, args, err in vr.cases(routine, device, "invalid"):
        with pytest.raises(wg.Error) as ei:
            vr.call(fn, args)
        assert err in str(ei.value), label
    n = 0
    for label, args, _ in vr.cases(routine, device, "edge"):
        assert result_key({"routine": routine}) in vr.call(fn, args), label
        n += 1
    assert n >= 10


def random_case(routine, side, uplo, layout, m, n, transA="no-transpose", diag="non-unit", pad=2, seed=1,
                alpha=0.5, beta=1.25):
    rng = np.random.default_rng(seed)
    dt = np.float64 if routine.startswith("d") else np.float32
    cm = layout == "column-major"
    order = m if side == "left" else n
    lda, ldb, ldc = order + pad, (m if cm else n) + pad, (m if cm else n) + pad
    outer = n if cm else m
    case = {"routine": routine, "side": side, "uplo": uplo, "layout": layout, "m": m, "n": n, "alpha": alpha,
            "A": (rng.random(lda * order) * 2 - 1).astype(dt), "lda": lda,
            "B": (rng.random(ldb * outer) * 2 - 1).astype(dt), "ldb": ldb}
    if routine.endswith("trmm"):
        case.update(transA=transA, diag=diag)
    else:
        case.update(beta=beta, C=(rng.random(ldc * outer) * 2 - 1).astype(dt), ldc=ldc)
    return case


def block_mask(case, ld):
    m, n = case["m"], case["n"]
    i, j = np.meshgrid(np.arange(m), np.arange(n), indexing="ij")
    idx = (j * ld + i) if case["layout"] == "column-major" else (i * ld + j)
    mask = np.zeros(case[result_key(case)].size, bool)
    mask[idx.ravel()] = True
    return mask, idx


def check_bound(case, got):
    """|got - truth| <= 2*K*2^-24 (f32) or 4*K*2^-53 (f64) times (|alpha||X||Y| + |beta||C|)."""
    f64 = case["routine"].startswith("d")
    m, n = case["m"], case["n"]
    D, order = dense_operand(case, np.float64)
    D = D.reshape(order, order, order="F")
    Bd = general(case, "B", case["ldb"], np.float64).reshape(m, n, order="F")
    X, Y = (D, Bd) if case["side"] == "left" else (Bd, D)
    truth = case["alpha"] * (X @ Y)
    scale = abs(case["alpha"]) * (np.abs(X) @ np.abs(Y))
    if not case["routine"].endswith("trmm"):
        Cd = general(case, "C", case["ldc"], np.float64).reshape(m, n, order="F")
        truth = truth + case["beta"] * Cd
        scale = scale + abs(case["beta"]) * np.abs(Cd)
    eps = 4 * 2.0**-53 if f64 else 2 * 2.0**-24
    ld = case["ldb"] if case["routine"].endswith("trmm") else case["ldc"]
    mask, idx = block_mask(case, ld)
    g = got[idx].astype(np.float64)
    assert np.all(np.abs(g - truth) <= eps * order * scale)
    src = case[result_key(case)]
    assert bits_equal(got[~mask], src[~mask]), "padding changed"


@pytest.mark.parametrize("routine", ROUTINES)
@pytest.mark.parametrize("side", ["left", "right"])
@pytest.mark.parametrize("uplo", ["lower", "upper"])
@pytest.mark.parametrize("layout", ["column-major", "row-major"])
def test_simt_bit_exact(wg, device, oracle, routine, side, uplo, layout):
    device.set_sgemm_path("simt")
    device.set_dgemm_path("simt")
    try:
        seed = ROUTINES.index(routine) * 8 + (side == "right") * 4 + (uplo == "upper") * 2 + (layout == "row-major")
        extra = {"transA": "transpose", "diag": "unit"} if routine.endswith("trmm") and seed % 2 else {}
        case = random_case(routine, side, uplo, layout, m=70, n=45, seed=seed, **extra)
        got = call(wg, device, case, case["A"], case["B"], case.get("C"))[result_key(case)]
    finally:
        device.set_sgemm_path("auto")
        device.set_dgemm_path("auto")
    assert bits_equal(got, restate(oracle, case, 1))


@pytest.mark.parametrize("routine", ROUTINES)
@pytest.mark.parametrize("side", ["left", "right"])
@pytest.mark.parametrize("layout", ["column-major", "row-major"])
def test_tensor_core_paths(wg, device, routine, side, layout):
    extra = {"transA": "transpose", "diag": "unit"} if routine.endswith("trmm") and side == "right" else {}
    case = random_case(routine, side, "lower" if layout == "row-major" else "upper", layout, m=520, n=600, seed=5,
                       **extra)
    got = call(wg, device, case, case["A"], case["B"], case.get("C"))[result_key(case)]
    check_bound(case, got)


def test_gpumatrix_in_place(wg, device, oracle):
    case = random_case("strmm", "left", "upper", "column-major", m=300, n=260, pad=0, seed=9)
    m, n = case["m"], case["n"]
    GA = wg.GpuMatrix.from_(device, case["A"], m, m, case["lda"], "column-major")
    GB = wg.GpuMatrix.from_(device, case["B"], m, n, case["ldb"], "column-major")
    try:
        r = wg.strmm(device, "left", "upper", "no-transpose", "non-unit", m, n, case["alpha"], GA, case["lda"], GB,
                     case["ldb"])
        assert "B" not in r
        got = GB.read()
    finally:
        GA.destroy()
        GB.destroy()
    check_bound(case, got)
    case = random_case("ssymm", "right", "lower", "row-major", m=200, n=330, pad=0, seed=10)
    m, n = case["m"], case["n"]
    GA = wg.GpuMatrix.from_(device, case["A"], n, n, case["lda"], "row-major")
    GB = wg.GpuMatrix.from_(device, case["B"], m, n, case["ldb"], "row-major")
    GC = wg.GpuMatrix.from_(device, case["C"], m, n, case["ldc"], "row-major")
    try:
        r = wg.ssymm(device, "right", "lower", m, n, case["alpha"], GA, case["lda"], GB, case["ldb"], case["beta"], GC,
                     case["ldc"])
        assert "C" not in r
        got = GC.read()
    finally:
        for g in (GA, GB, GC):
            g.destroy()
    check_bound(case, got)
