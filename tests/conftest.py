"""Shared fixtures. GPU tests are marked ``gpu``; everything else runs on CPU."""
from __future__ import annotations

import json
import math
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA (sm_100) device")


def _decode(v):
    if isinstance(v, str) and v in ("NaN", "Infinity", "-Infinity"):
        return {"NaN": math.nan, "Infinity": math.inf, "-Infinity": -math.inf}[v]
    if isinstance(v, list):
        return [_decode(x) for x in v]
    if isinstance(v, dict):
        return {k: _decode(x) for k, x in v.items()}
    return v


def load_golden(name, decode=True):
    """A fixture from tests/golden/; decode=True turns "NaN"/"Infinity" strings into floats."""
    with open(os.path.join(GOLDEN, name)) as fh:
        data = json.load(fh)
    return _decode(data) if decode else data


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as o

    o.build()
    return o


@pytest.fixture(scope="session")
def wg():
    import wgblas_b200

    return wgblas_b200


@pytest.fixture(scope="session")
def device(wg):
    """The primary CUDA device (a benchmark device, so calls also report gpuTimeMs)."""
    if wg._native.device_count() == 0:
        pytest.fail("GPU test run without a visible CUDA device")
    dev = wg.init(benchmark=True)
    yield dev
    wg.cleanup()


def bits_equal(a: np.ndarray, b: np.ndarray) -> bool:
    """Bit-for-bit equality (distinguishes -0 from +0; any NaN equals any NaN)."""
    a = np.asarray(a)
    b = np.asarray(b)
    if a.shape != b.shape or a.dtype != b.dtype:
        return False
    nan = np.isnan(a) & np.isnan(b)
    ia = a.view(np.uint32 if a.dtype == np.float32 else np.uint64)
    ib = b.view(np.uint32 if b.dtype == np.float32 else np.uint64)
    return bool(np.all((ia == ib) | nan))
