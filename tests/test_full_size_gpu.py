"""configs[4] at full size on one GPU: sgemm and dgemm 16384^3 NN, alpha = beta = 1,
A, B, C ~ U[-1,1] seeded, through the plain entry points (wg_sgemm / wg_dgemm on
resident buffers) and through the sharded path with a one-rank communicator
(the code that runs on every rank of the multi-GPU runs, minus the transfer).
The whole product runs on the GPU; sampled columns are checked against the
oracle's fp64 (sgemm) or long-double (dgemm) truth with the north-star bounds
(a full CPU product of this size would take hours). The reference itself
cannot hold a 16384^2 matrix in one binding (benchmarks/utils/harness.mjs:54-55)."""
from __future__ import annotations

import numpy as np
import pytest

from gemm_check import sampled_columns_truth

pytestmark = pytest.mark.gpu
N = 16384
COLS = np.unique(np.concatenate([[0, 1, N - 1], np.linspace(0, N - 1, 13).astype(int)]))


def _inputs(wg, f64):
    rnd = wg.randomFloat64Array if f64 else wg.randomFloat32Array
    return rnd(N * N, -1, 1, 61), rnd(N * N, -1, 1, 62), rnd(N * N, -1, 1, 63)


def _check(oracle, f64, A, B, C, got_cols):
    """got_cols: N x len(COLS) result columns; asserts the bound on every element."""
    truth, absab, Cs = sampled_columns_truth(oracle, f64, 0, 0, N, N, N, 1.0, A, N, B, N, 1.0, C, N, COLS)
    t = oracle.dense(truth, N, len(COLS))
    bound = (oracle.dgemm_bound if f64 else oracle.sgemm_bound)(N, len(COLS), N, 1.0, absab, 1.0, Cs, N)
    g = got_cols.astype(np.float64)
    assert np.all(np.isfinite(g))
    err = np.abs(g - t)
    ratio = float(np.max(err / np.where(bound > 0, bound, 1)))
    print(f"{'dgemm' if f64 else 'sgemm'} 16384^3: max err/bound {ratio:.3e}")
    assert np.all(err <= bound), f"max err/bound {ratio}"


def _columns(flat):
    return np.stack([flat[j * N:(j + 1) * N] for j in COLS], axis=1)


@pytest.mark.parametrize("f64", [False, True], ids=["sgemm", "dgemm"])
def test_config5_plain_entry_point(wg, device, oracle, f64):
    A, B, C = _inputs(wg, f64)
    GA = wg.GpuMatrix.from_(device, A, N, N, N, "column-major")
    GB = wg.GpuMatrix.from_(device, B, N, N, N, "column-major")
    GC = wg.GpuMatrix.from_(device, C, N, N, N, "column-major")
    try:
        fn = wg.dgemm if f64 else wg.sgemm
        fn(device, "no-transpose", "no-transpose", N, N, N, 1.0, GA, N, GB, N, 1.0, GC, N, "column-major")
        device.synchronize()
        device.check()
        got = GC.read()
    finally:
        for g in (GA, GB, GC):
            g.destroy()
    _check(oracle, f64, A, B, C, _columns(got))


@pytest.mark.parametrize("f64", [False, True], ids=["sgemm", "dgemm"])
def test_config5_sharded_one_rank(wg, device, oracle, f64):
    from wgblas_b200.shard import Comm, gemm_sharded

    A, B, C = _inputs(wg, f64)
    comm = Comm(device, 1, 0, Comm.unique_id(), timeout_ms=60000)
    GA = wg.GpuMatrix.from_(device, A, N, N, N, "column-major")
    GB = wg.GpuMatrix.from_(device, B, N, N, N, "column-major")
    GC = wg.GpuMatrix.from_(device, C, N, N, N, "column-major")
    try:
        gemm_sharded(comm, False, False, N, N, N, 1.0, GA, GB, 1.0, GC, root=0, ldb=N)
        device.synchronize()
        comm.wait()
        device.check()
        got = GC.read()
    finally:
        for g in (GA, GB, GC):
            g.destroy()
        comm.destroy()
    _check(oracle, f64, A, B, C, _columns(got))


def test_config5_sharded_host_arrays_one_rank(wg, device, oracle):
    """The host-array form of the sharded call (gemm_sharded_host) at a smaller
    shape with uneven panels: the result on the root is the full C."""
    from wgblas_b200.shard import Comm, gemm_sharded_host, plan_rows

    m, n, k = 1500, 1300, 700
    A = wg.randomFloat32Array(m * k, -1, 1, 71)
    B = wg.randomFloat32Array(k * n, -1, 1, 72)
    C = wg.randomFloat32Array(m * n, -1, 1, 73)
    comm = Comm(device, 1, 0, Comm.unique_id(), timeout_ms=60000)
    try:
        out = wg.pinned_empty(m * n, np.float32)
        got = gemm_sharded_host(comm, False, False, m, n, k, 0.5, A, B, k, -1.0, C, plan_rows(m, 1), out=out)
    finally:
        comm.destroy()
    assert got is out
    truth, absab = oracle.sgemm_truth(0, 0, m, n, k, 0.5, A, m, B, k, -1.0, C, m)
    bound = oracle.sgemm_bound(m, n, k, 0.5, absab, -1.0, C, m)
    err = np.abs(oracle.block(got, m, n, m).astype(np.float64) - oracle.dense(truth, m, n))
    assert np.all(err <= bound)
