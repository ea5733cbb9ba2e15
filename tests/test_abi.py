"""The C ABI library loads, exports every function include/wgblas.h declares,
and its host-only entry points behave. CPU only: no kernel is launched."""
from __future__ import annotations

import ctypes as ct
import os
import re

import numpy as np

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
