"""One rank of the sharded-GEMM GPU check (run by tests/test_shard_gpu.py under
torchrun, or in-process with world 1). Builds seeded inputs, keeps this rank's
row blocks resident, broadcasts B from rank 0 in panels with the sharded call,
gathers C on rank 0 and checks it against the CPU oracle's truth bound."""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def run(dev, comm, rank, world, routine, m, n, k, ta, tb, alpha, beta, panel):
    import wgblas_b200 as wg
    from oracle import oracle as o
    from wgblas_b200.shard import gather_rows, gemm_sharded, plan_rows, row_block

    f64 = routine == "dgemm"
    dt = np.float64 if f64 else np.float32
    rnd = wg.randomFloat64Array if f64 else wg.randomFloat32Array
    lda = (k if ta else m)
    ldb = (n if tb else k)
    A = rnd(lda * (m if ta else k), -1, 1, 101)
    B = rnd(ldb * (k if tb else n), -1, 1, 102)
    C = rnd(m * n, -1, 1, 103)
    offs = plan_rows(m, world)
    r0, r1 = offs[rank], offs[rank + 1]
    mr = r1 - r0
    A_loc, lda_loc = row_block(A, m, k, lda, r0, r1, bool(ta))
    C_loc, ldc_loc = row_block(C, m, n, m, r0, r1, False)
    a_rows, a_cols = (k, mr) if ta else (mr, k)
    GA = wg.GpuMatrix.from_(dev, A_loc, a_rows, a_cols, lda_loc, "column-major")
    GC = wg.GpuMatrix.from_(dev, C_loc, mr, n, ldc_loc, "column-major")
    b_rows, b_cols = (n, k) if tb else (k, n)
    # B on the root only; odd ranks pass none at all, even ones a zeroed matrix
    GB = (wg.GpuMatrix.from_(dev, B if rank == 0 else np.zeros_like(B), b_rows, b_cols, ldb, "column-major")
          if rank % 2 == 0 else None)
    GF = wg.GpuMatrix.empty(dev, m, n, m, "column-major", dt) if rank == 0 else None
    try:
        gemm_sharded(comm, ta, tb, mr, n, k, alpha, GA, GB, beta, GC, root=0, panel_cols=panel, ldb=ldb)
        comm.wait()
        gather_rows(comm, GC, mr, n, offs, root=0, C_full=GF)
        dev.synchronize()
        dev.check()
        if rank != 0:
            return True
        got = GF.read()
        tr = (o.dgemm_truth if f64 else o.sgemm_truth)(ta, tb, m, n, k, alpha, A, lda, B, ldb, beta, C, m)
        bound = (o.dgemm_bound if f64 else o.sgemm_bound)(m, n, k, alpha, tr[1], beta, C, m)
        err = np.abs(o.block(got, m, n, m).astype(np.float64) - o.dense(tr[0], m, n))
        ok = bool(np.all(err <= bound))
        print(f"rank0 {routine} {m}x{n}x{k} ta={ta} tb={tb} world={world}: max err/bound "
              f"{float(np.max(err / np.where(bound > 0, bound, 1))):.3e} ok={ok}", flush=True)
        return ok
    finally:
        for g in (GA, GB, GC, GF):
            if g is not None:
                g.destroy()


CASES = [("sgemm", 1000, 777, 300, 0, 0, 1.5, 0.5, 256), ("sgemm", 640, 512, 256, 1, 1, 1.0, 0.0, 0),
         ("sgemm", 1000, 2900, 640, 0, 0, 0.5, -1.0, 0),  # planned panels; uneven row blocks at world 2
         ("dgemm", 700, 333, 129, 0, 0, -0.75, 1.25, 100), ("dgemm", 384, 256, 64, 1, 0, 2.0, -1.0, 0)]


def main():
    import datetime

    import torch.distributed as dist

    import wgblas_b200 as wg
    from wgblas_b200.shard import comm_from_torch

    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    rank, world = dist.get_rank(), dist.get_world_size()
    dev = wg.init(device=local)
    comm = comm_from_torch(dev, timeout_ms=60000)
    ok = True
    try:
        for case in CASES:
            ok &= run(dev, comm, rank, world, *case)
            dist.barrier()
    finally:
        comm.destroy()
        wg.cleanup()
        dist.destroy_process_group()
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
