"""The row-sharded GEMM on GPUs: one rank on one GPU (the broadcast is a no-op
but the panel pipeline, events and gather all run), and two ranks under
torchrun when two GPUs are visible."""
from __future__ import annotations

import os
import subprocess
import sys

import pytest

import shard_worker

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("case", shard_worker.CASES, ids=lambda c: f"{c[0]}-{c[1]}x{c[2]}x{c[3]}")
def test_sharded_single_rank(wg, device, case):
    from wgblas_b200.shard import Comm

    comm = Comm(device, 1, 0, Comm.unique_id(), timeout_ms=30000)
    try:
        assert shard_worker.run(device, comm, 0, 1, *case)
    finally:
        comm.destroy()


def test_sharded_two_ranks(wg):
    if wg._native.device_count() < 2:
        pytest.skip("needs two GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29533",
           os.path.join(ROOT, "tests", "shard_worker.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=400)
    print(r.stdout[-3000:], r.stderr[-3000:])
    assert r.returncode == 0
