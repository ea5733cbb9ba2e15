"""Failure detection on the GPU without a fault: a kernel waits, with the same
clock-bounded mbarrier wait the tensor-core kernels use, on a barrier nothing
completes. The wait gives up after its budget, the kernel records the timeout
and returns, the host reads WG_ERR_KERNEL_TIMEOUT from wg_device_check, and the
context keeps working."""
from __future__ import annotations

import time

import pytest

from gemm_check import check_sgemm

pytestmark = pytest.mark.gpu
N = "no-transpose"


def test_bounded_wait_reports_timeout_and_context_survives(wg, device, oracle):
    nat = wg._native
    device.synchronize()
    t0 = time.perf_counter()
    nat.check(nat.lib.wg_selftest_bounded_wait(device.handle, 20000))  # 20 ms of SM clock
    st = nat.lib.wg_device_check(device.handle)
    waited = time.perf_counter() - t0
    assert st == nat.WG_ERR_KERNEL_TIMEOUT
    assert "bounded wait" in nat.lib.wg_last_error().decode()
    assert waited >= 0.01, waited  # the wait really ran for its budget
    # the word is cleared by the check, and the device still computes
    assert nat.lib.wg_device_check(device.handle) == nat.WG_OK
    m, n, k = 256, 320, 200
    A = wg.randomFloat32Array(m * k, -1, 1, 5)
    B = wg.randomFloat32Array(k * n, -1, 1, 6)
    C = wg.randomFloat32Array(m * n, -1, 1, 7)
    got = wg.sgemm(device, N, N, m, n, k, 1.0, A, m, B, k, 0.5, C, m, "column-major")["C"]
    check_sgemm(oracle, got, N, N, m, n, k, 1.0, A, m, B, k, 0.5, C, m, "column-major")


def test_bounded_wait_rejects_bad_budget(wg, device):
    nat = wg._native
    assert nat.lib.wg_selftest_bounded_wait(device.handle, 0) == nat.WG_ERR_INVALID_ARGUMENT
    assert nat.lib.wg_selftest_bounded_wait(device.handle, 2_000_000) == nat.WG_ERR_INVALID_ARGUMENT


def test_a_rank_that_leaves_between_steps(wg):
    """Two GPUs (skipped with fewer): rank 1 leaves after a sharded product;
    rank 0 learns of it from the store before its next launch, aborts its
    communicator without waiting on the departed rank, and keeps computing."""
    import os
    import subprocess
    import sys

    if wg._native.device_count() < 2:
        pytest.skip("needs two GPUs")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "180", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29541",
           os.path.join(root, "tests", "leave_worker.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=260)
    print(r.stdout[-3000:], r.stderr[-3000:])
    assert r.returncode == 0
    assert "rank 1 left" in r.stdout and "device still computes: True" in r.stdout
