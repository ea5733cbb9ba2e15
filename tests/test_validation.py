"""Argument validation of sgemm / dgemm against the reference's invalid-value
specs (tests/validation/params/*.json via tests/golden/validation_params.json).
CPU only: every invalid call must raise before any device work, so a stand-in
device whose handle must never be touched is enough."""
from __future__ import annotations

import numpy as np
import pytest

import validation_runner as vr



@pytest.fixture(scope="module")
def fake_device(wg):
    class Fake(wg.Device):
        __slots__ = ()

        @property
        def handle(self):
            raise AssertionError("validation reached a native call")

    return Fake(object(), 0, False, {}, "fake")


@pytest.mark.parametrize("routine", ["sgemm", "dgemm", "sgemmtr", "dgemmtr", "ssyrk", "dsyrk", "ssyr2k", "dsyr2k",
                                     "ssymm", "dsymm", "strmm", "dtrmm", "strsm", "sgemv", "dgemv"])
def test_invalid_arguments_raise_reference_messages(wg, fake_device, routine):
    fn = getattr(wg, routine)
    n = 0
    for label, args, err in vr.cases(routine, fake_device, "invalid"):
        with pytest.raises(wg.Error) as ei:
            vr.call(fn, args)
        assert err in str(ei.value), f"{label}: {ei.value!r} lacks {err!r}"
        n += 1
    assert n >= 40


def test_config4_illegal_ldb_is_rejected(wg, fake_device):
    """BASELINE config 4 with transB=T: B is stored n x k column-major, so ldb=800 < n=1023
    is rejected exactly as src/sgemm/sgemm.mjs:117-120 rejects it."""
    m, n, k = 1000, 1023, 777
    A = np.zeros(1024 * 1000, np.float32)
    B = np.zeros(800 * 1023, np.float32)
    C = np.zeros(1040 * 1023, np.float32)
    for ta in ("no-transpose", "transpose"):
        with pytest.raises(wg.Error, match="ldb must be >= rows of B as stored."):
            wg.sgemm(fake_device, ta, "transpose", m, n, k, 0.3, A, 1024, B, 800, -2.0, C, 1040,
                     "column-major")


def test_mixed_gpu_and_array_operands(wg, fake_device):
    class M(wg.GpuMatrix):
        def __init__(self):
            pass

    g = M()
    g.device = fake_device
    g.layout = "row-major"
    g.dtype = np.float32
    a = np.zeros(4, np.float32)
    with pytest.raises(wg.Error, match="C must be a GpuMatrix when A or B is a GpuMatrix."):
        wg.sgemm(fake_device, "no-transpose", "no-transpose", 2, 2, 2, 1, g, 2, a, 2, 0, a, 2)
    with pytest.raises(wg.Error, match="A and B must be GpuMatrix when C is a GpuMatrix."):
        wg.sgemm(fake_device, "no-transpose", "no-transpose", 2, 2, 2, 1, a, 2, a, 2, 0, g, 2)
    g.device = object()
    with pytest.raises(wg.Error, match="sgemm: A belongs to a different GPUDevice"):
        wg.sgemm(fake_device, "no-transpose", "no-transpose", 2, 2, 2, 1, g, 2, a, 2, 0, a, 2)


def test_zero_dims_return_input_unchanged(wg, fake_device):
    C = np.arange(4, dtype=np.float32)
    for m, n in ((0, 2), (2, 0)):
        r = wg.sgemm(fake_device, "no-transpose", "no-transpose", m, n, 2, 1, C, 2, C, 2, 0, C, 2)
        assert r["C"] is C


def test_dgemm_quick_return_is_the_same_array(wg, fake_device):
    A = np.ones(4)
    C = np.array([1 / 3, np.pi, -0.0, 5.0])
    for alpha, k in ((0.0, 2), (1.5, 0)):
        r = wg.dgemm(fake_device, "no-transpose", "no-transpose", 2, 2, k, alpha, A, 2, A, 2, 1, C, 2)
        assert r["C"] is C
