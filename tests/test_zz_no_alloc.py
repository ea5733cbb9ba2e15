"""wg_sgemm_noalloc: the sgemm entry point for callers that cannot allocate device
memory (their own allocator owns the GPU's memory, or an allocation's implicit
synchronisation is not allowed where they call from). It must give the same
result as the allocating entry point, wg_sgemm_dev on the same 3xTF32 kernel,
within the sgemm tolerance the other tests use, on consecutive calls sharing
its fixed scratch array. Collected last so a failure here comes after every
other test has run; it also passes alone in a fresh process."""
from __future__ import annotations

import ctypes as ct

import numpy as np
import pytest

from gemm_check import frame

pytestmark = pytest.mark.gpu
T, N = "transpose", "no-transpose"


def _dev_array(wg, dev, host):
    buf = ct.c_void_p()
    wg._native.check(wg._native.lib.wg_buffer_alloc(dev.handle, host.nbytes, ct.byref(buf)))
    wg._native.check(wg._native.lib.wg_buffer_upload(buf, 0, host.ctypes.data_as(ct.c_void_p), host.nbytes))
    ptr = ct.c_void_p()
    wg._native.check(wg._native.lib.wg_buffer_device_ptr(buf, ct.byref(ptr)))
    return buf, ptr


def _read(wg, buf, like):
    out = np.empty_like(like)
    wg._native.check(wg._native.lib.wg_buffer_download(buf, 0, out.ctypes.data_as(ct.c_void_p), out.nbytes))
    return out


def _one_call(wg, dev, oracle, ta, tb, m, n, k, alpha, beta, seed):
    L = wg._native.lib
    lda, ldb, ldc = (k if ta else m), (n if tb else k), m + 3
    A = wg.randomFloat32Array(lda * (m if ta else k), -1, 1, seed)
    B = wg.randomFloat32Array(ldb * (k if tb else n), -1, 1, seed + 1)
    C = wg.randomFloat32Array(ldc * n, -1, 1, seed + 2)
    bufs = []
    try:
        a, pa = _dev_array(wg, dev, A)
        b, pb = _dev_array(wg, dev, B)
        c1, pc1 = _dev_array(wg, dev, C)
        c2, pc2 = _dev_array(wg, dev, C)
        bufs = [a, b, c1, c2]
        wg._native.check(L.wg_sgemm_noalloc(dev.handle, ta, tb, m, n, k, alpha, pa, lda, pb, ldb, beta, pc1, ldc))
        dev.set_sgemm_path("tf32x3")
        try:
            wg._native.check(L.wg_sgemm_dev(dev.handle, ta, tb, m, n, k, alpha, pa, lda, pb, ldb, beta, pc2, ldc))
        finally:
            dev.set_sgemm_path("auto")
        dev.synchronize()
        dev.check()
        got, want = _read(wg, c1, C), _read(wg, c2, C)
    finally:
        for buf in bufs:
            L.wg_buffer_free(buf)
    truth, absab = oracle.sgemm_truth(ta, tb, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc)
    bound = oracle.sgemm_bound(m, n, k, alpha, absab, beta, C, ldc)
    g = oracle.block(got, m, n, ldc).astype(np.float64)
    w = oracle.block(want, m, n, ldc).astype(np.float64)
    assert np.all(np.abs(g - w) <= bound), "differs from the allocating entry point beyond the tolerance"
    assert np.all(np.abs(g - oracle.dense(truth, m, n)) <= bound)
    pad = np.ones(C.size, bool)
    for j in range(n):
        pad[j * ldc: j * ldc + m] = False
    assert np.array_equal(got[pad], C[pad]), "ldc padding was written"


def test_no_alloc_matches_allocating_entry_point(wg, device, oracle):
    # Two calls in a row sharing the scratch array, with different shapes and transposes.
    _one_call(wg, device, oracle, 1, 0, 512, 384, 256, 1.0, 0.0, 11)
    _one_call(wg, device, oracle, 0, 1, 300, 520, 1000, 1.5, -0.5, 21)


def test_no_alloc_rejects_oversized_problems(wg, device):
    L = wg._native.lib
    # 4096^3 needs 256 MiB of split-operand scratch, beyond the fixed 64 MiB.
    st = L.wg_sgemm_noalloc(device.handle, 0, 0, 4096, 4096, 4096, 1.0, ct.c_void_p(16), 4096, ct.c_void_p(16),
                            4096, 0.0, ct.c_void_p(16), 4096)
    assert st == wg._native.WG_ERR_INVALID_ARGUMENT
    assert b"scratch" in L.wg_last_error()


def test_no_alloc_calls_take_no_device_memory(wg, device):
    """The property the entry point exists for: after a handle is open, its calls
    reserve no device memory. A fresh handle (empty grow-only workspace) runs a
    shape whose allocating plan would split tiles along k (so falling back to
    the workspace path would show), and the GPU's free memory is unchanged
    across further calls."""
    import torch

    L = wg._native.lib
    dev = wg.init(powerPreference="high-performance", benchmark=False, device=device.ordinal)
    assert dev is not device
    plan = wg._native.TcPlan()
    wg._native.check(L.wg_sgemm_tc_plan(dev.props()["sm_count"], 1024, 1024, 2048, ct.byref(plan)))
    assert plan.split_segments > 1, "pick a shape whose allocating plan splits tiles"
    m = n = 1024
    k = 2048
    A = wg.randomFloat32Array(m * k, -1, 1, 31)
    B = wg.randomFloat32Array(k * n, -1, 1, 32)
    bufs = []
    try:
        a, pa = _dev_array(wg, dev, A)
        b, pb = _dev_array(wg, dev, B)
        c, pc = _dev_array(wg, dev, np.zeros(m * n, np.float32))
        bufs = [a, b, c]
        torch.cuda.mem_get_info(dev.ordinal)  # torch's own context first
        wg._native.check(L.wg_sgemm_noalloc(dev.handle, 0, 0, m, n, k, 1.0, pa, m, pb, k, 0.0, pc, m))
        dev.synchronize()
        free0, _ = torch.cuda.mem_get_info(dev.ordinal)
        for _ in range(2):
            wg._native.check(L.wg_sgemm_noalloc(dev.handle, 0, 0, m, n, k, 1.0, pa, m, pb, k, 0.5, pc, m))
        dev.synchronize()
        dev.check()
        free1, _ = torch.cuda.mem_get_info(dev.ordinal)
        assert free1 == free0, f"device memory changed by {free0 - free1} bytes"
    finally:
        for buf in bufs:
            L.wg_buffer_free(buf)
        wg.cleanup(dev)
