"""One rank of the "a rank leaves" GPU check (run by tests/test_failure_gpu.py
under torchrun on two GPUs, NVLS off). Both ranks run one sharded product; then
rank 1 leaves between steps, with none of its work in flight and without any
cleanup, as a crashed process would. Rank 0 learns of it on the host, from the
rendezvous store, before its next launch: it aborts its communicator, frees it,
and shows that its device still computes (an sgemm checked against the oracle).
No kernel or copy touches the departed rank's memory after it left."""
from __future__ import annotations

import datetime
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tests"))


def main():
    import torch.distributed as dist

    import shard_worker
    import wgblas_b200 as wg
    from oracle import oracle as o
    from wgblas_b200.shard import comm_from_torch

    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=30))
    rank, world = dist.get_rank(), dist.get_world_size()
    store = dist.distributed_c10d._get_default_store()
    dev = wg.init(device=local)
    comm = comm_from_torch(dev, timeout_ms=5000)
    ok = shard_worker.run(dev, comm, rank, world, "sgemm", 640, 512, 256, 0, 0, 1.0, 0.5, 0)
    dev.synchronize()
    if rank == 1:
        store.set("wgblas_rank1_left", "1")
        sys.stdout.flush()
        os._exit(0)
    t0 = time.perf_counter()
    store.wait(["wgblas_rank1_left"], datetime.timedelta(seconds=20))
    comm.abort()
    comm.destroy()
    noticed = time.perf_counter() - t0
    m, n, k = 300, 260, 150
    A = wg.randomFloat32Array(m * k, -1, 1, 21)
    B = wg.randomFloat32Array(k * n, -1, 1, 22)
    C = wg.randomFloat32Array(m * n, -1, 1, 23)
    got = wg.sgemm(dev, "no-transpose", "no-transpose", m, n, k, 1.0, A, m, B, k, 0.5, C, m, "column-major")["C"]
    truth, absab = o.sgemm_truth(0, 0, m, n, k, 1.0, A, m, B, k, 0.5, C, m)
    bound = o.sgemm_bound(m, n, k, 1.0, absab, 0.5, C, m)
    ok &= bool(np.all(np.abs(o.block(got, m, n, m).astype(np.float64) - o.dense(truth, m, n)) <= bound))
    wg.cleanup()
    print(f"rank0: rank 1 left; communicator aborted and freed {noticed:.2f} s later; "
          f"device still computes: {ok}", flush=True)
    os._exit(0 if ok else 1)  # the process group's peer is gone: no collective teardown


if __name__ == "__main__":
    main()
