"""The kernel-path switches across the boundary (CPU): every WG_SGEMM_* code of
include/wgblas.h has the same value in the ctypes table and a name in
Device.set_sgemm_path, and the C ABI accepts exactly those codes."""
from __future__ import annotations

import ctypes as ct
import os
import re

from conftest import ROOT


def _header_codes(prefix):
    text = open(os.path.join(ROOT, "include", "wgblas.h")).read()
    return {m.group(1): int(m.group(2)) for m in re.finditer(r"#define (" + prefix + r"\w+) (\d+)", text)}


def test_sgemm_codes_match_the_header(wg):
    from wgblas_b200._runtime import SGEMM_PATHS

    codes = _header_codes("WG_SGEMM_")
    assert codes, "no WG_SGEMM_ codes in the header"
    for name, value in codes.items():
        assert getattr(wg._native, name) == value, name
    assert sorted(SGEMM_PATHS.values()) == sorted(codes.values())


def test_sgemm_path_range_is_checked(wg):
    N = wg._native
    block = (ct.c_char * 65536)()  # a zeroed stand-in for a device handle; the setter only stores the code
    dev = ct.cast(block, ct.c_void_p)
    for value in _header_codes("WG_SGEMM_").values():
        assert N.lib.wg_device_set_sgemm_path(dev, value) == N.WG_OK
    for bad in (-1, max(_header_codes("WG_SGEMM_").values()) + 1):
        assert N.lib.wg_device_set_sgemm_path(dev, bad) == N.WG_ERR_INVALID_ARGUMENT
        assert "unknown sgemm path" in N.lib.wg_last_error().decode()
