"""The C ABI library loads, exports every function include/wgblas.h declares,
and its host-only entry points behave. CPU only: no kernel is launched."""
from __future__ import annotations

import ctypes as ct
import os
import re

import numpy as np
import pytest

from conftest import ROOT, bits_equal, load_golden


def _declared():
    with open(os.path.join(ROOT, "include", "wgblas.h")) as fh:
        text = fh.read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(wg_[a-z0-9_]+)\s*\(", text)))


def test_every_declared_symbol_is_exported(wg):
    lib = wg._native.lib
    names = _declared()
    assert len(names) >= 30
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_abi_version(wg):
    assert wg._native.lib.wg_abi_version() == 1


def test_device_count_reports_without_error(wg):
    n = ct.c_int(-1)
    assert wg._native.lib.wg_device_count(ct.byref(n)) == 0
    assert n.value >= 0


def test_null_arguments_are_rejected(wg):
    L = wg._native.lib
    assert L.wg_device_open(0, 0, None) == wg._native.WG_ERR_INVALID_ARGUMENT
    assert L.wg_sgemm(None, 0, 0, 1, 1, 1, 1.0, None, 0, 1, None, 0, 1, 0.0, None, 0, 1, None) == \
        wg._native.WG_ERR_INVALID_ARGUMENT
    assert b"NULL" in L.wg_last_error()
    assert L.wg_dgemm_host(None, 0, 0, 1, 1, 1, 1.0, None, 1, None, 1, 0.0, None, None, 1, None) == \
        wg._native.WG_ERR_INVALID_ARGUMENT


def test_open_without_device_reports_no_device(wg):
    if wg._native.device_count() == 0:
        h = ct.c_void_p()
        assert wg._native.lib.wg_device_open(0, 0, ct.byref(h)) == wg._native.WG_ERR_NO_DEVICE


def test_library_random_matches_oracle_and_golden(wg, oracle):
    g = load_golden("mulberry32.json")
    for seed, draws in g["seeds"].items():
        assert list(wg.randomFloat64Array(16, 0, 1, int(seed))) == draws
    for seed in (0, 1, 100, 111, 200, 300):
        assert bits_equal(wg.randomFloat32Array(1000, -1, 1, seed), oracle.random_f32(1000, -1, 1, seed))
        assert bits_equal(wg.randomFloat64Array(1000, -5, 5, seed), oracle.random_f64(1000, -5, 5, seed))
        assert bits_equal(wg.randomNormalFloat32Array(1001, seed), oracle.normal_f32(1001, seed))
        assert bits_equal(wg.randomNormalFloat64Array(1001, seed), oracle.normal_f64(1001, seed))


def test_unseeded_random_differs(wg):
    a, b = wg.randomFloat32Array(64), wg.randomFloat32Array(64)
    assert not np.array_equal(a, b) and a.min() >= -1 and a.max() < 1


def test_every_declared_function_has_a_binding(wg):
    """_native declares argument and result types for every entry point, so no
    call goes through ctypes' int defaults."""
    lib = wg._native.lib
    unbound = [n for n in _declared() if getattr(lib, n).argtypes is None]
    assert not unbound, unbound


def test_null_device_is_rejected_by_the_level3_and_level2_entry_points(wg):
    L, N = wg._native.lib, wg._native
    bad = N.WG_ERR_INVALID_ARGUMENT
    assert L.wg_strsm(None, 0, 1, 0, 0, 2, 2, 1.0, None, 0, 2, None, 0, 2, None) == bad
    assert L.wg_strsm_dev(None, 0, 1, 0, 0, 2, 2, 1.0, None, 2, None, 2) == bad
    assert L.wg_sgemv(None, 0, 2, 2, 1.0, None, 0, 2, None, 0, 1, 0.0, None, 0, 1, None) == bad
    assert L.wg_dgemv(None, 1, 2, 2, 1.0, None, 0, 2, None, 0, 1, 0.0, None, 0, 1, None) == bad
    assert L.wg_sgemv_dev(None, 0, 2, 2, 1.0, None, 2, None, 1, 0.0, None, 1) == bad
    assert L.wg_symmetrize(None, 4, 1, 2, None, 0, 2, None, 0, 2) == bad
    assert L.wg_triangularize(None, 8, 2, 0, 1, 2, None, 0, 2, None, 0, 2) == bad
    h = N.c_buf_p()
    assert L.wg_buffer_alloc_async(None, 64, ct.byref(h)) == bad
    assert b"NULL" in L.wg_last_error() or b"invalid" in L.wg_last_error()


def _blank_device():
    """A zeroed block standing in for a device handle: the argument checks of the
    entry points below run before any field is read, and a zero compute
    capability then stops them with WG_ERR_NOT_SUPPORTED, before any CUDA call."""
    block = (ct.c_char * 65536)()
    return block, ct.cast(block, ct.c_void_p)


@pytest.mark.parametrize("args,status,text", [
    ((2, 1, 0, 0, 4, 3, 4, 4), "INVALID_ARGUMENT", "side must be"),
    ((0, 0, 0, 0, 4, 3, 4, 4), "INVALID_ARGUMENT", "uplo must be"),
    ((0, 1, 2, 0, 4, 3, 4, 4), "INVALID_ARGUMENT", "transA must be"),
    ((0, 1, 0, 2, 4, 3, 4, 4), "INVALID_ARGUMENT", "diag must be"),
    ((0, 1, 0, 0, -1, 3, 4, 4), "INVALID_ARGUMENT", "m and n must be non-negative."),
    ((0, 1, 0, 0, 4, 3, 0, 4), "INVALID_ARGUMENT", "lda and ldb must be positive."),
    ((0, 1, 0, 0, 4, 3, 3, 4), "INVALID_ARGUMENT", "lda must be >= m."),
    ((1, 1, 0, 0, 4, 3, 2, 4), "INVALID_ARGUMENT", "lda must be >= n."),
    ((0, 1, 0, 0, 4, 3, 4, 3), "INVALID_ARGUMENT", "ldb must be >= rows of B as stored."),
    ((0, 1, 0, 0, 0, 3, 1, 1), "OK", ""),
    ((0, 2, 1, 1, 4, 3, 4, 4), "NOT_SUPPORTED", "not a Blackwell"),
])
def test_strsm_argument_checks(wg, args, status, text):
    N = wg._native
    keep, dev = _blank_device()
    side, uplo, trans, diag, m, n, lda, ldb = args
    st = N.lib.wg_strsm_dev(dev, side, uplo, trans, diag, m, n, 1.0, None, lda, None, ldb)
    assert st == getattr(N, "WG_" + status if status == "OK" else "WG_ERR_" + status)
    if text:
        assert text in N.lib.wg_last_error().decode()


@pytest.mark.parametrize("args,status,text", [
    ((2, 4, 3, 4, 1, 1), "INVALID_ARGUMENT", "trans must be"),
    ((0, -1, 3, 4, 1, 1), "INVALID_ARGUMENT", "m and n must be non-negative."),
    ((0, 4, 3, 4, 0, 1), "INVALID_ARGUMENT", "incx and incy must be positive."),
    ((1, 4, 3, 4, 1, -2), "INVALID_ARGUMENT", "incx and incy must be positive."),
    ((0, 4, 3, 0, 1, 1), "INVALID_ARGUMENT", "lda must be positive."),
    ((0, 4, 3, 3, 1, 1), "INVALID_ARGUMENT", "lda must be >= rows of A as stored."),
    ((0, 4, 0, 1, 1, 1), "OK", ""),
    ((1, 4, 3, 5, 2, 3), "NOT_SUPPORTED", "not a Blackwell"),
])
def test_gemv_argument_checks(wg, args, status, text):
    N = wg._native
    keep, dev = _blank_device()
    trans, m, n, lda, incx, incy = args
    for fn in (N.lib.wg_sgemv_dev, N.lib.wg_dgemv_dev):
        st = fn(dev, trans, m, n, 1.0, None, lda, None, incx, 0.5, None, incy)
        assert st == getattr(N, "WG_" + status if status == "OK" else "WG_ERR_" + status)
        if text:
            assert text in N.lib.wg_last_error().decode()
