"""Host logic of the row-sharded multi-GPU GEMM on CPU: row planning, the
row-block extraction and reassembly, and the broadcast/gather choreography,
run as two gloo ranks (world_size 2) with the oracle standing in for each
rank's GPU GEMM — the reassembled C must equal the single-process oracle
result bit for bit. Also: a rank that leaves makes the other rank's next
collective fail within the process-group timeout instead of hanging."""
from __future__ import annotations

import os
import socket
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_plan_rows_covers_and_aligns():
    from wgblas_b200.shard import plan_rows

    for m in (0, 1, 127, 128, 1000, 16384, 16385):
        for p in (1, 2, 3, 4, 8):
            offs = plan_rows(m, p)
            assert offs[0] == 0 and offs[-1] == m and len(offs) == p + 1
            sizes = np.diff(offs)
            assert np.all(sizes >= 0)
            for r in range(p):
                if offs[r + 1] < m:
                    assert sizes[r] % 128 == 0, (m, p, offs)
            assert sizes.max() - sizes.min() <= 256, (m, p, offs)


@pytest.mark.parametrize("trans", [False, True])
def test_row_block_roundtrip(trans):
    from wgblas_b200.shard import place_rows, row_block

    rng = np.random.default_rng(1)
    m, k, ld = 37, 11, 40
    X = rng.standard_normal(ld * (m if trans else k)).astype(np.float32)
    blk, ldb = row_block(X, m, k, ld, 5, 20, trans)
    for i in range(15):
        for p in range(k):
            want = X[p + (5 + i) * ld] if trans else X[(5 + i) + p * ld]
            got = blk[p + i * ldb] if trans else blk[i + p * ldb]
            assert got == want
    C = np.zeros(50 * 7, np.float32)
    place_rows(C, 50, np.arange(15 * 7, dtype=np.float32), 15, 5, 20, 7)
    assert C[5] == 0 and C[5 + 50] == 15


def _worker(rank, world, port, case, q):
    import datetime

    import torch
    import torch.distributed as dist

    sys.path.insert(0, ROOT)
    from oracle import oracle as o
    from wgblas_b200.shard import place_rows, plan_rows, row_block

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    try:
        m, n, k, ta, tb, alpha, beta = case
        rng = np.random.default_rng(7)  # same seed: every rank builds the same full inputs
        lda = (k if ta else m) + 1
        ldb = (n if tb else k) + 2
        A = rng.uniform(-1, 1, lda * (m if ta else k)).astype(np.float32)
        B_root = rng.uniform(-1, 1, ldb * (k if tb else n)).astype(np.float32)
        C = rng.uniform(-1, 1, m * n).astype(np.float32)
        offs = plan_rows(m, world, align=16)
        r0, r1 = offs[rank], offs[rank + 1]
        A_loc, lda_loc = row_block(A, m, k, lda, r0, r1, ta)
        C_loc, ldc_loc = row_block(C, m, n, m, r0, r1, False)
        # the broadcast of B from root (the NCCL broadcast of the GPU path)
        B = torch.from_numpy(B_root.copy() if rank == 0 else np.zeros_like(B_root))
        dist.broadcast(B, src=0)
        B = B.numpy()
        out = o.sgemm(ta, tb, r1 - r0, n, k, alpha, A_loc, lda_loc, B, ldb, beta, C_loc, ldc_loc, variant=1) \
            if r1 > r0 else C_loc
        blocks = [None] * world
        dist.all_gather_object(blocks, (r0, r1, out, ldc_loc))
        if rank == 0:
            full = C.copy()
            for (a0, a1, blk, ldbk) in blocks:
                place_rows(full, m, blk, ldbk, a0, a1, n)
            want = o.sgemm(ta, tb, m, n, k, alpha, A, lda, B_root, ldb, beta, C, m, variant=1)
            q.put(bool(np.array_equal(full.view(np.uint32), want.view(np.uint32))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("case", [(70, 33, 19, 0, 0, 1.5, 0.5), (45, 64, 40, 1, 1, -0.75, 1.25),
                                  (17, 9, 5, 1, 0, 2.0, 0.0)])
def test_sharded_two_ranks_reassemble_exactly(case):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    mp.start_processes(_worker, args=(2, _free_port(), case, q), nprocs=2, join=True, start_method="spawn")
    assert q.get(timeout=5) is True


def _leaver(rank, world, port, q):
    import datetime

    import torch
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    if rank == 1:
        os._exit(0)  # leaves between steps, with nothing in flight
    t = torch.zeros(4)
    try:
        dist.broadcast(t, src=1)
        q.put("no error")
    except Exception as e:  # noqa: BLE001
        q.put(type(e).__name__)


def test_rank_that_leaves_surfaces_as_error():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_leaver, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=60)
    assert all(not p.is_alive() for p in procs)
    assert q.get(timeout=5) != "no error"
