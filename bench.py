#!/usr/bin/env python
"""Benchmark of the sgemm/dgemm hot path on B200 — prints ONE JSON line.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload W]

Metric: sgemm/dgemm TFLOP/s and % of FP32/FP64 peak, FLOPs
counted as the reference counts them, 2*m*n*k + 2*m*n
(benchmarks/sgemm/wgblas/sgemm.js:72-73).

Workloads:
  sgemm4096   configs[1]: sgemm 4096^3 column-major TN, alpha=1, beta=0, A,B ~ N(0,1), C=0
              (the default at N=1)
  sgemm2048   sgemm 2048^3 NN, U[-1,1] (a mid-size shape for profiling single kernels)
  dgemm2048   the same for dgemm
  dgemm4096   configs[2]: dgemm 4096^3 column-major NT, alpha=-0.75, beta=1.25, U[-1,1]
  sgemm512    configs[0]: sgemm 512^3 NN, alpha=1.5, beta=0.5, U[-1,1]
  ragged      configs[3]: sgemm 1000x1023x777, lda=1024 ldb=800 ldc=1040, NN
  shard16384  configs[4]: sgemm 16384^3 NN, alpha=1, beta=1, U[-1,1], C row-block sharded
              over the ranks with B broadcast from rank 0 over NVLink (the default at N>1)
  shard16384d the same for dgemm
A step is one sgemm/dgemm call on operands resident in HBM; L2 is flushed
(a 512 MB device write) between steps, outside the per-step CUDA events.
With --gpus N>1 (torchrun) the default workload is shard16384: each rank keeps
its row block of A and C resident, and every step broadcasts B from rank 0 in
column panels (the library's planned widths for sgemm, one panel for dgemm),
each panel's GEMM overlapping the next panel's transfer;
value = total FLOPs / max over ranks of the step time (strong scaling).

At N=1 the line's "extra" also carries the other configs and the next routines
at the reference's benchmark shapes (gemmtr/syrk, symm/trmm, strsm, gemv), each
with "routine", "shape" and "ms_per_step" for the roofline report
(python -m wgblas_b200.roofline), the roofline probes of the run, and a cuBLAS
column (torch.mm at 4096^3, fp32 with TF32 off and fp64) for comparison.

--impl reference times the reference's arithmetic on the host cores instead:
the CPU oracle's restatement of the reference's fp32 shader arithmetic
(oracle/, "port"; the reference itself runs only through WebGPU, which has no
stack on these boxes), on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
METRIC = "sgemm/dgemm TFLOP/s & % of FP32/FP64 peak at 4096³ (1 GPU), 16384³ at 1/2/4/8"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}

WORKLOADS = {
    "sgemm4096": dict(routine="sgemm", config_index=1, transA=1, transB=0, m=4096, n=4096, k=4096,
                      lda=4096, ldb=4096, ldc=4096, alpha=1.0, beta=0.0, data="normal"),
    "dgemm4096": dict(routine="dgemm", config_index=2, transA=0, transB=1, m=4096, n=4096, k=4096,
                      lda=4096, ldb=4096, ldc=4096, alpha=-0.75, beta=1.25, data="uniform"),
    "sgemm512": dict(routine="sgemm", config_index=0, transA=0, transB=0, m=512, n=512, k=512,
                     lda=512, ldb=512, ldc=512, alpha=1.5, beta=0.5, data="uniform"),
    "ragged": dict(routine="sgemm", config_index=3, transA=0, transB=0, m=1000, n=1023, k=777,
                   lda=1024, ldb=800, ldc=1040, alpha=0.3, beta=-2.0, data="uniform"),
    "shard16384": dict(routine="sgemm", config_index=4, transA=0, transB=0, m=16384, n=16384, k=16384,
                       lda=16384, ldb=16384, ldc=16384, alpha=1.0, beta=1.0, data="uniform", sharded=True),
    "shard16384d": dict(routine="dgemm", config_index=4, transA=0, transB=0, m=16384, n=16384, k=16384,
                        lda=16384, ldb=16384, ldc=16384, alpha=1.0, beta=1.0, data="uniform", sharded=True),
    "sgemm2048": dict(routine="sgemm", config_index=None, transA=0, transB=0, m=2048, n=2048, k=2048,
                      lda=2048, ldb=2048, ldc=2048, alpha=1.0, beta=0.5, data="uniform"),
    "dgemm2048": dict(routine="dgemm", config_index=None, transA=0, transB=0, m=2048, n=2048, k=2048,
                      lda=2048, ldb=2048, ldc=2048, alpha=1.0, beta=0.5, data="uniform"),
    # The gemmtr family at the reference's own benchmark shape (benchmarks/sgemmtr/wgblas/sgemmtr.js,
    # benchmarks/ssyrk/wgblas/ssyrk.js: m = n = k, lower, alpha 1, beta 0), counted as it counts them.
    "sgemmtr4096": dict(routine="sgemm", config_index=None, transA=0, transB=0, m=4096, n=4096, k=4096,
                        lda=4096, ldb=4096, ldc=4096, alpha=1.0, beta=0.0, data="uniform", uplo=1),
    "ssyrk4096": dict(routine="sgemm", config_index=None, transA=0, transB=1, m=4096, n=4096, k=4096,
                      lda=4096, ldb=4096, ldc=4096, alpha=1.0, beta=0.0, data="uniform", uplo=1, syrk=True),
    "dsyrk4096": dict(routine="dgemm", config_index=None, transA=0, transB=1, m=4096, n=4096, k=4096,
                      lda=4096, ldb=4096, ldc=4096, alpha=1.0, beta=0.0, data="uniform", uplo=1, syrk=True),
}
PANEL_COLS = 0  # B broadcast panels of the sharded workloads: 0 = the library's plan
# DRAM traffic of one launch of the dominant kernel (dram__bytes_read.sum +
# dram__bytes_write.sum, bytes) from the ncu capture of the same kernel and
# workload summarised in profiles/ (tests/test_bench_traffic.py keeps these in
# step with those files).
NCU_TRAFFIC = {
    ("sgemm4096", "sgemm_tf32x3_mma"): (626.0e6, 61.7e6, "profiles/sgemm_tf32x3_4096_TN.md"),
    ("dgemm4096", "dgemm_dmma"): (1233.8e6, 122.7e6, "profiles/dgemm_dmma_4096_NT.md"),
}


def flops(w):
    if w.get("uplo"):  # the triangle only: k multiply-adds for each of n(n+1)/2 elements
        return float(w["n"]) * (w["n"] + 1) * w["k"]
    return 2.0 * w["m"] * w["n"] * w["k"] + 2.0 * w["m"] * w["n"]


def stored(w):
    a = (w["k"], w["m"]) if w["transA"] else (w["m"], w["k"])
    b = (w["n"], w["k"]) if w["transB"] else (w["k"], w["n"])
    return a, b


def host_inputs(wg, w, pinned=False):
    """Seeded column-major operands at the workload's leading dimensions."""
    (ar, ac), (br, bc) = stored(w)
    dt = np.float64 if w["routine"] == "dgemm" else np.float32
    sizes = (w["lda"] * ac, w["ldb"] * bc, w["ldc"] * w["n"])
    out = []
    for seed, size in zip((1, 2, 3), sizes):
        arr = wg.pinned_empty(size, dt) if pinned else np.empty(size, dt)
        if w["data"] == "normal" and seed != 3:
            (wg.randomNormalFloat64Array if dt == np.float64 else wg.randomNormalFloat32Array)(size, seed, out=arr)
        elif w["data"] == "normal":
            arr[:] = 0
        else:
            wg.fill_uniform(arr, -1.0, 1.0, seed)
        out.append(arr)
    return out


class L2Flush:
    """Evicts the operands from the 126 MB L2 between timed steps: ``add_`` writes a
    512 MB buffer (the flush the timing rule names), then reads a 256 MB one, so
    that the dirty lines the write leaves in L2 go back to HBM here, outside the
    timed region, instead of inside the next step (where an HBM-bound kernel
    would pay for them)."""

    def __init__(self, device):
        import torch

        self.w = torch.empty(128 * 1024 * 1024, dtype=torch.float32, device=device)
        self.r = torch.zeros(64 * 1024 * 1024, dtype=torch.float32, device=device)

    def add_(self, value):
        import torch

        self.w.add_(value)
        torch.sum(self.r)


class Clocks:
    """Samples SM clocks and throttle reasons with nvidia-smi during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        rows = []
        try:
            with open(self.path) as fh:
                for line in fh:
                    parts = [p.strip() for p in line.split(",")]
                    if len(parts) >= 9 and parts[1].replace(".", "").isdigit():
                        rows.append(parts)
        finally:
            os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        sm = [float(r[1]) for r in rows]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": float(rows[0][2]), "reasons": reasons,
                "samples": len(rows), "power_w_max": max(float(r[3]) for r in rows if r[3].replace(".", "").isdigit())}


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as fh:
            return json.load(fh), "measured (MEASURED_PEAKS.json)"
    return FALLBACK_PEAKS, "fallback (profiling recipe)"


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
    return world, rank, local


def max_over_ranks(x, world):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([float(x)], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x, world):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist

    t = torch.tensor([float(x)], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


PARITY_COLS = 16  # sampled columns of C checked after the timed region


def parity_columns(w, m_rows, A, lda, B, C0, ldc, got, ldg, ncols=PARITY_COLS):
    """Checks sampled columns of one result against the fp64 truth (numpy only).

    A is this rank's op(A) source (column-major, ``lda``; ``m_rows`` rows of
    op(A)), B the full stored B (ld = w["ldb"]), C0 the C the checked call
    started from (column-major, ld ``ldc``) and got the C it left (ld ``ldg``). The bound is
    the north star's: |got - truth| <= 2*K*2^-24*(|alpha| sum|a||b| + |beta||c|)
    for sgemm, 4*K*2^-53*(...) for dgemm. The truth is numpy's fp64 product,
    whose own error (at most K*2^-53 of the same sum) counts against the
    measured one, so a pass is never looser than the stated bound allows."""
    k, n = w["k"], w["n"]
    ta, tb = w["transA"], w["transB"]
    cols = np.unique(np.linspace(0, n - 1, ncols).astype(np.int64))
    if ta:
        opA = A[: m_rows * lda].reshape(m_rows, lda)[:, :k]
    else:
        opA = A[: k * lda].reshape(k, lda)[:, :m_rows].T
    ldb = w["ldb"]
    if tb:
        Bs = np.stack([B[j + np.arange(k) * ldb] for j in cols], axis=1)
    else:
        Bs = np.stack([B[j * ldb: j * ldb + k] for j in cols], axis=1)
    Cs = np.stack([C0[j * ldc: j * ldc + m_rows] for j in cols], axis=1).astype(np.float64)
    Gs = np.stack([got[j * ldg: j * ldg + m_rows] for j in cols], axis=1).astype(np.float64)
    A64 = opA.astype(np.float64)
    B64 = Bs.astype(np.float64)
    alpha, beta = float(w["alpha"]), float(w["beta"])
    truth = alpha * (A64 @ B64) + beta * Cs
    np.abs(A64, out=A64)
    absab = abs(alpha) * (A64 @ np.abs(B64)) + abs(beta) * np.abs(Cs)
    del A64
    unit = 2.0 * k * 2.0 ** -24 if w["routine"] == "sgemm" else 4.0 * k * 2.0 ** -53
    bound = unit * absab
    err = np.abs(Gs - truth)
    finite = bool(np.all(np.isfinite(Gs)))
    ratio = float(np.max(err / np.where(bound > 0, bound, 1.0))) if err.size else 0.0
    return {"ok": bool(finite and np.all(err <= bound)), "max_err_over_bound": ratio,
            "cols": int(len(cols)), "rows": int(m_rows),
            "bound": "2*K*2^-24*(|alpha|sum|a||b|+|beta||c|)" if w["routine"] == "sgemm"
            else "4*K*2^-53*(|alpha|sum|a||b|+|beta||c|)",
            "truth": "numpy fp64 product of the sampled columns"}


def parity_over_ranks(par, world):
    """Every rank's parity folded into one record: ok on all ranks, the worst ratio."""
    if world == 1:
        return par
    ok = min_over_ranks(1.0 if par["ok"] else 0.0, world) > 0.5
    ratio = max_over_ranks(par["max_err_over_bound"], world)
    out = dict(par, ok=ok, max_err_over_bound=ratio, ranks=world)
    out["rows"] = int(sum_over_ranks(par["rows"], world))
    return out


def min_over_ranks(x, world):
    return -max_over_ranks(-float(x), world)


def gemm_enqueue(wg, dev, w, GA, GB, GC):
    """One step on resident operands, queued on the device stream (no host sync)."""
    nat = wg._native
    if w.get("uplo"):
        # gemmtr; syrk is gemmtr with B := A and the other transpose, as ssyrk composes it
        fn = nat.lib.wg_dgemmtr if w["routine"] == "dgemm" else nat.lib.wg_sgemmtr
        B, ldb = (GA, w["lda"]) if w.get("syrk") else (GB, w["ldb"])
        nat.check(fn(dev.handle, w["uplo"], w["transA"], w["transB"], w["m"], w["n"], w["k"], w["alpha"], GA._buf, 0,
                     w["lda"], B._buf, 0, ldb, w["beta"], GC._buf, 0, w["ldc"], None))
        return
    fn = nat.lib.wg_dgemm if w["routine"] == "dgemm" else nat.lib.wg_sgemm
    nat.check(fn(dev.handle, w["transA"], w["transB"], w["m"], w["n"], w["k"], w["alpha"], GA._buf, 0, w["lda"],
                 GB._buf, 0, w["ldb"], w["beta"], GC._buf, 0, w["ldc"], None))


def time_resident(wg, dev, w, steps, warmup, world, flush, parity=True):
    """Device-timed steps on resident operands: returns (ms_per_step list, profile,
    launches, wall seconds, parity). The per-kernel events (profile) come from a
    second pass of the same flushed steps right after the timed one: recorded
    between a call's launches they lengthen the step (12 us of a 49 us configs[3]
    call), and they would break the programmatic overlap of consecutive launches.
    After that, C is restored, one more call runs, and sampled columns of its
    result are checked against the fp64 truth (parity_columns)."""
    import torch

    from wgblas_b200.classes import _upload

    A, B, C = host_inputs(wg, w)
    (ar, ac), (br, bc) = stored(w)
    GA = wg.GpuMatrix.from_(dev, A, ar, ac, w["lda"], "column-major")
    GB = wg.GpuMatrix.from_(dev, B, br, bc, w["ldb"], "column-major")
    GC = wg.GpuMatrix.from_(dev, C, w["m"], w["n"], w["ldc"], "column-major")
    stream = torch.cuda.ExternalStream(dev.stream(), device=torch.device("cuda", dev.ordinal))
    try:
        with torch.cuda.stream(stream):
            for _ in range(warmup):
                flush.add_(1.0)
                gemm_enqueue(wg, dev, w, GA, GB, GC)
            dev.synchronize()
            dev.check()
            starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
            ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
            barrier(world)
            dev.synchronize()
            dev.profile_read()
            launches0 = dev.kernel_launches()
            t0 = time.perf_counter()
            for i in range(steps):
                flush.add_(1.0)  # evicts the operands from the 126 MB L2 (L2Flush)
                starts[i].record(stream)
                gemm_enqueue(wg, dev, w, GA, GB, GC)
                ends[i].record(stream)
            dev.synchronize()
            wall = time.perf_counter() - t0
            launches = dev.kernel_launches() - launches0
            dev.check()
            ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
            dev.set_profiling(True)  # per-kernel events, in a pass of its own
            for _ in range(steps):
                flush.add_(1.0)
                gemm_enqueue(wg, dev, w, GA, GB, GC)
            dev.synchronize()
            dev.set_profiling(False)
            prof = dev.profile_read()
            dev.check()
            par = None
            if parity:
                _upload(GC._buf, C[: w["ldc"] * w["n"]])
                gemm_enqueue(wg, dev, w, GA, GB, GC)
                dev.synchronize()
                dev.check()
                got = GC.read()
                if w.get("uplo"):
                    par = None  # the gemmtr lines: parity lives in the tests (triangle semantics)
                else:
                    par = parity_columns(w, w["m"], A, w["lda"], B, C, w["ldc"], got, w["m"])
    finally:
        for g in (GA, GB, GC):
            g.destroy()
    return ms, prof, launches, wall, par


def time_special(wg, dev, name, steps, warmup, flush):
    """ssymm / strmm at 4096 (the reference's benchmark defaults: side left, uplo
    lower, trmm non-unit no-transpose; benchmarks/ssymm/wgblas/ssymm.js,
    benchmarks/strmm/wgblas/strmm.js) through the public API on resident
    GpuMatrix operands, with the reference's FLOP counts."""
    import torch

    n = 4096
    A = wg.randomFloat32Array(n * n, -1, 1, 1)
    B = wg.randomFloat32Array(n * n, -1, 1, 2)
    GA = wg.GpuMatrix.from_(dev, A, n, n, n, "column-major")
    GB = wg.GpuMatrix.from_(dev, B, n, n, n, "column-major")
    GC = wg.GpuMatrix.from_(dev, wg.randomFloat32Array(n * n, -1, 1, 3), n, n, n, "column-major")
    if name == "ssymm4096":
        fn = lambda: wg.ssymm(dev, "left", "lower", n, n, 1.0, GA, n, GB, n, 0.0, GC, n, "column-major")  # noqa: E731
        work = 2.0 * n * n * n + 2.0 * n * n
    else:
        fn = lambda: wg.strmm(dev, "left", "lower", "no-transpose", "non-unit", n, n, 1.0, GA, n, GB, n, "column-major")  # noqa: E731
        work = 2.0 * n * n * n + 1.0 * n * n
    stream = torch.cuda.ExternalStream(dev.stream(), device=torch.device("cuda", dev.ordinal))
    try:
        with torch.cuda.stream(stream):
            for _ in range(warmup):
                flush.add_(1.0)
                fn()
            dev.synchronize()
            starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
            ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
            for i in range(steps):
                flush.add_(1.0)
                starts[i].record(stream)
                fn()
                ends[i].record(stream)
            dev.synchronize()
            ms = statistics.mean(s.elapsed_time(e) for s, e in zip(starts, ends))
    finally:
        for g in (GA, GB, GC):
            g.destroy()
    return {"tflops": work / (ms * 1e-3) / 1e12, "ms_per_step": ms, "routine": name[:5],
            "shape": {"m": n, "n": n, "aOrder": n},
            "note": "public API call incl. its scratch allocation and the dense operand pass"}


def time_trsm(wg, dev, nrhs, steps, warmup, flush):
    """strsm at order 4096, side left, lower, no-transpose, non-unit, column-major,
    through the public API on resident GpuMatrix operands. nrhs = 64 is the
    reference's base sweep (benchmarks/strsm/wgblas/strsm.js, order 4096 with a
    64-column right-hand side); nrhs = 4096 a square solve. B is refreshed from
    a pristine copy before every call, outside the timed events, as the
    reference's benchmark refreshes it (the solve is in place). A: off-diagonals
    in [-1/order, 1/order), diagonal in [5, 15) (diagonally dominant, so repeated
    solves stay finite). FLOPs: m*n*order (the reference's count)."""
    import ctypes as ct

    import torch

    from wgblas_b200 import _native as nat

    order = 4096
    rng = np.random.default_rng(4)
    A = ((rng.random(order * order) * 2 - 1) / order).astype(np.float32)
    A[np.arange(order) * (order + 1)] = (5 + 10 * rng.random(order)).astype(np.float32)
    B = wg.randomFloat32Array(order * nrhs, -1, 1, 2)
    GA = wg.GpuMatrix.from_(dev, A, order, order, order, "column-major")
    GB = wg.GpuMatrix.from_(dev, B, order, nrhs, order, "column-major")
    G0 = wg.GpuMatrix.from_(dev, B, order, nrhs, order, "column-major")
    pitch = order * 4

    def refresh():
        nat.check(nat.lib.wg_buffer_copy_2d(dev.handle, G0._buf, 0, pitch, GB._buf, 0, pitch, pitch, nrhs))

    def solve():
        wg.strsm(dev, "left", "lower", "no-transpose", "non-unit", order, nrhs, 1.0, GA, order, GB, order,
                 "column-major")

    stream = torch.cuda.ExternalStream(dev.stream(), device=torch.device("cuda", dev.ordinal))
    try:
        with torch.cuda.stream(stream):
            for _ in range(warmup):
                flush.add_(1.0)
                refresh()
                solve()
            dev.synchronize()
            starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
            ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
            for i in range(steps):
                flush.add_(1.0)
                refresh()
                starts[i].record(stream)
                solve()
                ends[i].record(stream)
            dev.synchronize()
            ms = statistics.mean(s.elapsed_time(e) for s, e in zip(starts, ends))
            x = GB.read()
    finally:
        for g in (GA, GB, G0):
            g.destroy()
    work = float(order) * nrhs * order
    return {"tflops": work / (ms * 1e-3) / 1e12, "ms_per_step": ms, "ms_per_block": ms / (order // 64),
            "finite": bool(np.all(np.isfinite(x))), "routine": "strsm",
            "shape": {"m": order, "n": nrhs, "aOrder": order},
            "note": "order 4096 left lower column-major; public API on GpuMatrix, B refreshed untimed"}


def time_gemv(wg, dev, routine, trans, steps, warmup, flush):
    """sgemv / dgemv at 4096 x 4096, column-major A, unit strides (the layout of
    the reference's base sweep, benchmarks/sgemv/wgblas/sgemv.js) on GpuMatrix
    and GpuVector operands: the public API once, then each timed step queues the
    C-ABI call it makes (wg_sgemv / wg_dgemv) without the host wait the public
    call adds after it.

    L2: inputs larger than L2. Four copies of A (256 / 512 MiB together) are
    used in turn, so the A a step reads was evicted by the three read since;
    the steps run back to back between one pair of events (the rate of a stream
    of calls; events between the steps add their own gaps). A second pass
    flushes L2 (the bench's write-then-read flush) before every step instead and
    is reported beside it: there the step also pays the launch and first-touch
    latency that back-to-back calls overlap (an empty kernel measures about 6 us
    in that setting). Bytes: A once, x once, y read and written (the reference's
    count); the HBM roof is the run's bandwidth probe."""
    import torch

    n = 4096
    dt = np.float64 if routine == "dgemv" else np.float32
    rnd = wg.randomFloat64Array if dt == np.float64 else wg.randomFloat32Array
    host_a = rnd(n * n, -1, 1, 1)
    GAs = [wg.GpuMatrix.from_(dev, host_a, n, n, n, "column-major") for _ in range(4)]
    gx = wg.GpuVector.from_(dev, rnd(n, -1, 1, 2))
    gy = wg.GpuVector.from_(dev, rnd(n, -1, 1, 3))
    fn = getattr(wg, routine)
    nat = wg._native
    cfn = nat.lib.wg_dgemv if dt == np.float64 else nat.lib.wg_sgemv
    t = 0 if trans == "no-transpose" else 1  # the column-major frame of this call (A column-major)

    def enqueue(i):  # the public call's C-ABI step, queued without a host wait
        nat.check(cfn(dev.handle, t, n, n, 1.0, GAs[i % 4]._buf, 0, n, gx._buf, 0, 1, 0.5, gy._buf, 0, 1, None))

    steps = max(steps, 20)
    stream = torch.cuda.ExternalStream(dev.stream(), device=torch.device("cuda", dev.ordinal))

    def events():
        return [torch.cuda.Event(enable_timing=True) for _ in range(steps)]

    try:
        with torch.cuda.stream(stream):
            fn(dev, trans, n, n, 1.0, GAs[0], n, gx, 1, 0.5, gy, 1)  # the public API once (validation, result)
            for i in range(max(warmup, 4)):
                enqueue(i)
            dev.synchronize()
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record(stream)
            for i in range(steps):  # back to back over the four copies
                enqueue(i)
            end.record(stream)
            dev.synchronize()
            ms = start.elapsed_time(end) / steps
            starts, ends = events(), events()
            for i in range(steps):  # flushed before every step
                flush.add_(1.0)
                starts[i].record(stream)
                enqueue(i)
                ends[i].record(stream)
            dev.synchronize()
            ms_flushed = statistics.mean(a.elapsed_time(b) for a, b in zip(starts, ends))
            dev.profile_read()
            dev.set_profiling(True)  # per-kernel events, in a pass of its own
            for i in range(steps):
                enqueue(i)
            dev.synchronize()
            dev.set_profiling(False)
            prof = dev.profile_read()
    finally:
        for g in (*GAs, gx, gy):
            g.destroy()
    item = np.dtype(dt).itemsize
    nbytes = (n * n + 3 * n) * item
    kernels = {k: v[1] / max(v[0], 1) for k, v in prof.items()}
    return {"gbs": nbytes / (ms * 1e-3) / 1e9, "tflops": 2.0 * n * n / (ms * 1e-3) / 1e12, "ms_per_step": ms,
            "routine": routine, "shape": {"m": n, "n": n, "trans": trans}, "kernels": kernels,
            "kernel_gbs": nbytes / (sum(kernels.values()) * 1e-3) / 1e9 if kernels else None,
            "flushed": {"ms_per_step": ms_flushed, "gbs": nbytes / (ms_flushed * 1e-3) / 1e9},
            "l2": "inputs larger than L2 (4 copies of A used in turn, K steps back to back between one event "
                  "pair); 'flushed' = L2 flushed before each step, events around each step",
            "note": "4096x4096 column-major A, unit strides; GpuMatrix/GpuVector operands: the public API once, "
                    "then the same C-ABI call queued per step without a host wait"}


def time_cublas(dt, steps, warmup, flush, local):
    """The library-GEMM comparison column of the reference's build plan: torch.mm
    (cuBLAS) at 4096^3 on the same GPU, fp32 with TF32 off (the FP32 SIMT path,
    the accuracy class of sgemm) or fp64, L2 flushed between steps. Not part of
    the product; reported beside it."""
    import torch

    n = 4096
    device = torch.device("cuda", local)
    torch_dt = torch.float64 if dt == "f64" else torch.float32
    g = torch.Generator(device=device).manual_seed(5)
    A = torch.rand((n, n), generator=g, device=device, dtype=torch_dt) * 2 - 1
    B = torch.rand((n, n), generator=g, device=device, dtype=torch_dt) * 2 - 1
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        for _ in range(warmup):
            flush.add_(1.0)
            C = torch.mm(A, B)
        torch.cuda.synchronize(device)
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        for i in range(steps):
            flush.add_(1.0)
            starts[i].record()
            C = torch.mm(A, B)
            ends[i].record()
        torch.cuda.synchronize(device)
        ms = statistics.mean(s.elapsed_time(e) for s, e in zip(starts, ends))
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    del A, B, C
    return {"tflops": 2.0 * n ** 3 / (ms * 1e-3) / 1e12, "ms_per_step": ms,
            "note": f"torch.mm (cuBLAS) {n}^3 {'fp64' if dt == 'f64' else 'fp32, TF32 off'}; comparison only"}


def sharded_inputs(wg, w, world, rank):
    """This rank's seeded row blocks of op(A) and C (dense column-major, ld = its
    rows) and the full B (generated on every rank: the root uploads it, the
    others use it only to check their result)."""
    from wgblas_b200.shard import plan_rows

    m, n, k = w["m"], w["n"], w["k"]
    offs = plan_rows(m, world)
    mr = offs[rank + 1] - offs[rank]
    dt = np.float64 if w["routine"] == "dgemm" else np.float32
    rnd = wg.randomFloat64Array if dt == np.float64 else wg.randomFloat32Array
    return offs, mr, rnd(mr * k, -1, 1, 10 + rank), rnd(k * n, -1, 1, 2), rnd(mr * n, -1, 1, 30 + rank)


def time_sharded(wg, dev, comm, w, steps, warmup, world, rank, flush, parity=True):
    """Device-timed steps of the row-sharded GEMM (B broadcast + local GEMMs).
    After the timed region every rank restores its C rows, one more sharded call
    runs, and each rank checks sampled columns of its rows against the fp64
    truth (parity_columns); the record is folded over the ranks."""
    import torch

    from wgblas_b200.classes import _upload
    from wgblas_b200.shard import gemm_sharded

    m, n, k = w["m"], w["n"], w["k"]
    offs, mr, A, B, C0 = sharded_inputs(wg, w, world, rank)
    GA = wg.GpuMatrix.from_(dev, A, mr, k, mr, "column-major")
    GC = wg.GpuMatrix.from_(dev, C0, mr, n, mr, "column-major")
    # B lives on the root only; the other ranks receive it into the library's buffer.
    GB = wg.GpuMatrix.from_(dev, B, k, n, k, "column-major") if rank == 0 else None
    stream = torch.cuda.ExternalStream(dev.stream(), device=torch.device("cuda", dev.ordinal))

    def step():
        gemm_sharded(comm, w["transA"], w["transB"], mr, n, k, w["alpha"], GA, GB, w["beta"], GC, root=0,
                     panel_cols=PANEL_COLS, ldb=k)

    try:
        with torch.cuda.stream(stream):
            for _ in range(warmup):
                flush.add_(1.0)
                step()
            dev.synchronize()
            comm.wait()
            dev.check()
            starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
            ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
            barrier(world)
            dev.synchronize()
            dev.profile_read()
            dev.set_profiling(True)
            launches0 = dev.kernel_launches()
            t0 = time.perf_counter()
            for i in range(steps):
                flush.add_(1.0)
                starts[i].record(stream)
                step()
                ends[i].record(stream)
            dev.synchronize()
            comm.wait()
            wall = time.perf_counter() - t0
            launches = dev.kernel_launches() - launches0
            dev.set_profiling(False)
            prof = dev.profile_read()
            dev.check()
            ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
            par = None
            if parity:
                _upload(GC._buf, C0)
                barrier(world)
                step()
                dev.synchronize()
                comm.wait()
                dev.check()
                par = parity_columns(w, mr, A, mr, B, C0, mr, GC.read(), mr)
                par = parity_over_ranks(par, world)
    finally:
        for g in (GA, GB, GC):
            if g is not None:
                g.destroy()
    return ms, prof, launches, wall, par


def time_e2e(wg, dev, w, steps, warmup):
    """The same metric through the public API on page-locked host arrays: every step
    uploads op(A), op(B) (and C when beta != 0), computes, and reads C back."""
    A, B, C = host_inputs(wg, w, pinned=True)
    out = wg.pinned_empty(C.size, C.dtype)
    fn = wg.dgemm if w["routine"] == "dgemm" else wg.sgemm
    tA = "transpose" if w["transA"] else "no-transpose"
    tB = "transpose" if w["transB"] else "no-transpose"
    args = (tA, tB, w["m"], w["n"], w["k"], w["alpha"], A, w["lda"], B, w["ldb"], w["beta"], C, w["ldc"],
            "column-major")
    for _ in range(max(1, warmup // 2)):
        fn(dev, *args, out=out)
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        fn(dev, *args, out=out)
        times.append(time.perf_counter() - t0)
    (ar, ac), (br, bc) = stored(w)
    item = C.dtype.itemsize
    h2d = (ar * ac + br * bc + (w["m"] * w["n"] if w["beta"] != 0 else 0)) * item
    d2h = w["m"] * w["n"] * item
    sec = statistics.mean(times)
    return {"value": flops(w) / sec / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": int(h2d),
            "d2h_bytes_per_step": int(d2h), "ms_per_step": sec * 1e3, "api": f"wgblas_b200.{w['routine']}"}


def time_e2e_sharded(wg, dev, comm, w, steps, warmup, world, rank):
    """The sharded metric end to end through the public host-array call
    (wgblas_b200.shard.gemm_sharded_host): every step each rank uploads its row
    blocks of op(A) and C from page-locked host memory, the root uploads B, the
    product runs sharded, C is gathered on the root and read back into a
    page-locked array. Timed with CUDA events on each rank's device stream
    around the whole call; the step time is the max over ranks."""
    import torch

    from wgblas_b200.shard import gemm_sharded_host

    m, n, k = w["m"], w["n"], w["k"]
    offs, mr, A, B, C0 = sharded_inputs(wg, w, world, rank)
    dt = A.dtype

    def pinned(x):
        p = wg.pinned_empty(x.size, dt)
        p[:] = x
        return p

    Ap, Cp = pinned(A), pinned(C0)
    Bp = pinned(B) if rank == 0 else None
    del A, B, C0
    out = wg.pinned_empty(m * n, dt) if rank == 0 else None
    stream = torch.cuda.ExternalStream(dev.stream(), device=torch.device("cuda", dev.ordinal))

    def call():
        gemm_sharded_host(comm, w["transA"], w["transB"], mr, n, k, w["alpha"], Ap, Bp, k, w["beta"], Cp, offs,
                          root=0, panel_cols=PANEL_COLS, out=out)

    for _ in range(max(1, warmup // 2)):
        call()
    times = []
    for _ in range(steps):
        barrier(world)
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        call()
        t1.record(stream)
        t1.synchronize()
        times.append(t0.elapsed_time(t1))
    ms = max_over_ranks(statistics.mean(times), world)
    item = np.dtype(dt).itemsize
    h2d = (m * k + m * n + k * n) * item
    return {"value": flops(w) / (ms * 1e-3) / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": int(h2d),
            "d2h_bytes_per_step": int(m * n * item), "ms_per_step": ms,
            "api": "wgblas_b200.shard.gemm_sharded_host",
            "timing": "CUDA events on each rank's device stream around the whole call, max over ranks"}


def cpu_baseline(w, target_s=12.0):
    """The oracle's restatement of the reference's arithmetic on the host cores, on a
    slab of C's columns sized for about target_s seconds, scaled to TFLOP/s."""
    sys.path.insert(0, ROOT)
    from oracle import oracle as o

    o.build()
    threads = o.default_threads()
    (ar, ac), (br, bc) = stored(w)
    m, k = w["m"], w["k"]
    dt = np.float64 if w["routine"] == "dgemm" else np.float32
    rng = np.random.default_rng(0)
    A = rng.random(w["lda"] * ac, dtype=dt) * 2 - 1

    def run(ns):
        B = rng.random(w["ldb"] * (ns if not w["transB"] else bc), dtype=dt) * 2 - 1
        ldb = w["ldb"]
        C = np.zeros(w["ldc"] * ns, dt)
        t0 = time.perf_counter()
        if w["routine"] == "dgemm":
            o.dgemm_dd(w["transA"], w["transB"], m, ns, k, w["alpha"], A, w["lda"], B, ldb, w["beta"], C, w["ldc"],
                       threads=threads)
        else:
            o.sgemm(w["transA"], w["transB"], m, ns, k, w["alpha"], A, w["lda"], B, ldb, w["beta"], C, w["ldc"],
                    variant=1, threads=threads)
        return time.perf_counter() - t0

    ns = max(1, min(w["n"], threads))
    t = run(ns)
    while t < 1.0 and ns < w["n"]:
        ns = min(w["n"], ns * 4)
        t = run(ns)
    if t < target_s and ns < w["n"]:
        ns = min(w["n"], max(ns, int(ns * target_s / max(t, 1e-3))))
        t = run(ns)
    f = 2.0 * m * ns * k + 2.0 * m * ns
    kind = "double-double restatement" if w["routine"] == "dgemm" else "fp32 FMA restatement"
    return {"value": f / t / 1e12, "unit": "TFLOP/s", "cores": threads, "kind": "port",
            "sample": f"{ns} of {w['n']} columns of C ({m}x{ns}x{k}), {kind} of the reference's shader "
                      f"arithmetic (oracle/oracle.c), {t:.1f} s", "seconds": t}


def run_reference(args, world, rank):
    """The reference arm: the oracle's restatement of the reference's arithmetic on
    the host cores (rank 0 only), each step a column slab of the same workload.
    ms_per_step is the time of the slab actually computed; value is the slab's
    FLOPs over that time (the sample names the slab). Nothing of wgblas_b200 is
    imported on this path."""
    if rank != 0:
        return 0
    w = WORKLOADS[pick_workload(args, world)]
    vals, secs = [], []
    cb = None
    for i in range(args.warmup + args.steps):
        cb = cpu_baseline(w, target_s=max(2.0, 60.0 / (args.warmup + args.steps)))
        if i >= args.warmup:
            vals.append(cb["value"])
            secs.append(cb["seconds"])
    value = statistics.mean(vals)
    line = {"metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": statistics.mean(secs) * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None,
            "dtype": "f64 (double-double)" if w["routine"] == "dgemm" else "f32",
            "data": "synthetic (seeded mulberry32)", "impl": "reference",
            "config": config_of(w, args.workload, world),
            "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": cb["cores"], "kind": "port",
                             "sample": cb["sample"] + "; each step computes this slab, ms_per_step is its time"},
            "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    emit(line)
    return 0


def pick_workload(args, world):
    if args.workload == "auto":
        return "shard16384" if world > 1 else "sgemm4096"
    return args.workload


def panel_plan(wg, w, world):
    """The broadcast panel widths a sharded call uses (its planned widths on the
    3xTF32 path; a dgemm product is one panel)."""
    if w["routine"] == "dgemm" or PANEL_COLS:
        return [w["n"]] if not PANEL_COLS else f"{PANEL_COLS} wide"
    import ctypes as ct

    import torch

    nat = wg._native
    sms = torch.cuda.get_device_properties(0).multi_processor_count if torch.cuda.is_available() else 148
    m_local = -(-w["m"] // world)
    widths = (ct.c_int64 * 4096)()
    count = ct.c_size_t()
    nat.check(nat.lib.wg_sharded_panel_plan(sms, world, m_local, w["n"], w["k"], widths, 4096, ct.byref(count)))
    return [int(widths[i]) for i in range(count.value)]


def routine_of(w):
    """The reference routine a workload times (the roofline tool's FLOP and byte counts)."""
    prefix = w["routine"][0]
    if w.get("syrk"):
        return prefix + "syrk"
    return prefix + "gemmtr" if w.get("uplo") else w["routine"]


def shape_of(w):
    return {"m": w["m"], "n": w["n"], "k": w["k"]}


def config_of(w, name, world=1):
    """The workload's description; identical on both arms (it reads nothing of the library)."""
    shard = ""
    if w.get("sharded"):
        shard = (f", C row-block sharded over {world} GPU(s), B broadcast from rank 0 over NVLink in "
                 "column panels")
    label = f"configs[{w['config_index']}]" if w.get("config_index") is not None else name
    return {"workload": f"{label} {w['routine']} {w['m']}x{w['n']}x{w['k']} "
                        f"{'T' if w['transA'] else 'N'}{'T' if w['transB'] else 'N'} column-major{shard}",
            "parallelism": f"row-sharded x{world}" if w.get("sharded") else "single GPU",
            "m": w["m"], "n": w["n"], "k": w["k"], "lda": w["lda"], "ldb": w["ldb"], "ldc": w["ldc"],
            "alpha": w["alpha"], "beta": w["beta"], "inputs": "N(0,1) seeded" if w["data"] == "normal" else "U[-1,1] seeded",
            "l2": "flushed between steps outside the step events (a 512 MB device write, then a 256 MB read "
                  "that writes the dirty lines back)",
            "routine": routine_of(w), "shape": shape_of(w),
            "scaling_note": ("N=1 times configs[1] (4096^3 sgemm); N>1 times configs[4] (16384^3, strong "
                             "scaling); extra.efficiency_same_config compares each N>1 value with the same "
                             "configuration on one GPU timed in the same run")}


_JSON_OUT = None


def emit(line: dict) -> None:
    """Writes the one JSON line to the process's original stdout."""
    out = _JSON_OUT if _JSON_OUT is not None else sys.stdout
    out.write(json.dumps(line) + "\n")
    out.flush()


def secondary(extra, key, fn):
    """Runs one secondary line; any failure is recorded under its key instead of
    costing the JSON line."""
    try:
        extra[key] = fn()
    except Exception as e:  # noqa: BLE001 (a secondary line must not cost the JSON line)
        extra[key] = {"error": f"{type(e).__name__}: {e}"}


def resident_line(wg, dev, wx, steps, flush, fp32_peak, fp64_peak):
    msx, profx, _, _, parx = time_resident(wg, dev, wx, steps, 3, 1, flush)
    tf = flops(wx) / (statistics.mean(msx) * 1e-3) / 1e12
    pk = fp64_peak if wx["routine"] == "dgemm" else fp32_peak
    line = {"tflops": tf, "ms_per_step": statistics.mean(msx), "routine": routine_of(wx), "shape": shape_of(wx),
            f"pct_of_{'fp64' if wx['routine'] == 'dgemm' else 'fp32'}_peak": 100.0 * tf / pk if pk else None,
            "kernels": {k: v[1] / max(v[0], 1) for k, v in profx.items()}}
    if parx is not None:
        line["parity"] = parx
    return line


def one_gpu_sharded_line(wg, dev, name, flush, fp32_peak, fp64_peak):
    """configs[4] on one GPU through the same sharded path (a one-rank
    communicator): the same-config reference point of the multi-GPU runs."""
    from wgblas_b200.shard import Comm

    ws = WORKLOADS[name]
    c1 = Comm(dev, 1, 0, Comm.unique_id())
    try:
        ms1, prof1, _, _, par1 = time_sharded(wg, dev, c1, ws, 3, 3, 1, 0, flush)
    finally:
        c1.destroy()
    tf1 = flops(ws) / (statistics.mean(ms1) * 1e-3) / 1e12
    pk = fp64_peak if ws["routine"] == "dgemm" else fp32_peak
    return {"tflops": tf1, "ms_per_step": statistics.mean(ms1), "routine": ws["routine"], "shape": shape_of(ws),
            f"pct_of_{'fp64' if ws['routine'] == 'dgemm' else 'fp32'}_peak": 100.0 * tf1 / pk if pk else None,
            "kernels": {k: v[1] / max(v[0], 1) for k, v in prof1.items()}, "parity": par1}


def main():
    # Native libraries (NCCL's banner, for one) may print to file descriptor 1;
    # move it to stderr for the whole run so stdout carries only the JSON line.
    global _JSON_OUT
    sys.stdout.flush()
    _JSON_OUT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--workload", choices=["auto"] + sorted(WORKLOADS), default="auto")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-extra", action="store_true", help="skip the secondary workloads and probes")
    p.add_argument("--sgemm-path", default="auto",
                   help="force an sgemm kernel (Device.set_sgemm_path: simt, simt_small, tf32x3, tf32x3_packed, "
                        "tf32x3_fused_bn256/128/64, tf32x3_pair) for profiling one kernel; the default picks by "
                        "shape")
    p.add_argument("--dgemm-path", default="auto", help="force a dgemm kernel (simt or dmma) for profiling")
    p.add_argument("--shape", default=None, metavar="M,N,K[,TA,TB]",
                   help="time one sgemm of this shape instead of a named workload (column-major, tight leading "
                        "dimensions, alpha 1.5, beta 0.5, U[-1,1] seeded; TA/TB 1 = transposed)")
    args = p.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.shape:
        dims = [int(x) for x in args.shape.split(",")]
        m, n, k = dims[:3]
        ta, tb = (dims[3], dims[4]) if len(dims) == 5 else (0, 0)
        WORKLOADS["shape"] = dict(routine="sgemm", config_index=None, transA=ta, transB=tb, m=m, n=n, k=k,
                                  lda=k if ta else m, ldb=n if tb else k, ldc=m, alpha=1.5, beta=0.5,
                                  data="uniform")
        args.workload = "shape"
    world, rank, local = dist_setup()
    if args.impl == "reference":
        return run_reference(args, world, rank)

    import torch

    sys.path.insert(0, ROOT)
    import wgblas_b200 as wg

    dev = wg.init(device=local)
    dev.set_sgemm_path(args.sgemm_path)
    dev.set_dgemm_path(args.dgemm_path)
    torch.cuda.set_device(local)
    wname = pick_workload(args, world)
    w = WORKLOADS[wname]
    flush = L2Flush(f"cuda:{local}")

    phys = os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",")
    smi_index = phys[local] if len(phys) > local and phys[local].strip() else str(local)
    comm = None
    if w.get("sharded"):
        from wgblas_b200.shard import Comm, comm_from_torch

        comm = comm_from_torch(dev) if world > 1 else Comm(dev, 1, 0, Comm.unique_id())
    with Clocks(smi_index) as clk:
        if w.get("sharded"):
            ms, prof, launches, wall, parity = time_sharded(wg, dev, comm, w, args.steps, args.warmup, world, rank,
                                                            flush)
        else:
            ms, prof, launches, wall, parity = time_resident(wg, dev, w, args.steps, args.warmup, world, flush)
            parity = parity_over_ranks(parity, world) if parity else parity
    clocks = clk.summary()
    step_ms = statistics.mean(ms)
    step_ms_max = max_over_ranks(step_ms, world)
    # sharded: the ranks together do one product; replicas: each rank does one
    value = flops(w) * (1 if w.get("sharded") else world) / (step_ms_max * 1e-3) / 1e12
    launches_total = int(sum_over_ranks(launches, world))

    peaks, peak_src = measured_peaks()
    extra = {}
    fp32_peak = fp64_peak = hbm = None
    short = max(3, args.steps // 2)
    if not args.no_extra and rank == 0:
        fp32_peak = dev.probe_peak("fp32")
        fp64_dfma = dev.probe_peak("fp64")
        fp64_dmma = dev.probe_peak("fp64_dmma")
        fp64_peak = max(fp64_dfma, fp64_dmma)  # the FP64 peak: the faster of the two FP64 pipes
        hbm = dev.probe_peak("hbm")
        extra["probes"] = {"fp32_ffma_tflops": fp32_peak, "fp64_dfma_tflops": fp64_dfma,
                           "fp64_dmma_tflops": fp64_dmma, "hbm_copy_gbs": hbm,
                           "source": "wg_probe_peak (benchmarks/roofline counterpart), this run"}
        extra["pct_of_fp32_peak"] = 100.0 * value / world / fp32_peak if w["routine"] == "sgemm" else None
        if world == 1:
            for name in ("dgemm4096", "sgemm512", "ragged", "sgemmtr4096", "ssyrk4096", "dsyrk4096"):
                if name != wname:
                    secondary(extra, name, lambda n=name: resident_line(wg, dev, WORKLOADS[n], short, flush,
                                                                        fp32_peak, fp64_peak))

    if not args.no_extra and world == 1 and not w.get("sharded"):
        for name in ("ssymm4096", "strmm4096"):
            secondary(extra, name, lambda n=name: time_special(wg, dev, n, short, 3, flush))
        for nrhs in (64, 4096):
            secondary(extra, f"strsm4096_n{nrhs}", lambda r=nrhs: time_trsm(wg, dev, r, short, 3, flush))
        # configs[4] on one GPU, sgemm and dgemm: the same-config reference points of the scaling runs.
        for name in ("shard16384", "shard16384d"):
            secondary(extra, f"{name}_1gpu", lambda n=name: one_gpu_sharded_line(wg, dev, n, flush, fp32_peak,
                                                                                 fp64_peak))
    if world > 1 and not args.no_extra and w["routine"] == "sgemm":
        # configs[4] for dgemm on the same ranks, with its parity
        wd = WORKLOADS["shard16384d"]
        msd, _, _, _, pard = time_sharded(wg, dev, comm, wd, 3, 3, world, rank, flush)
        md = max_over_ranks(statistics.mean(msd), world)
        extra["shard16384d"] = {"tflops": flops(wd) / (md * 1e-3) / 1e12, "ms_per_step": md, "parity": pard}
    if world > 1 and not args.no_extra and w.get("sharded"):
        # The same configuration on one GPU (rank 0, a one-rank communicator) in this
        # run, so that the scaling efficiency compares one workload with itself.
        one = {}
        if rank == 0:
            for name in (wname, "shard16384d") if w["routine"] == "sgemm" else (wname,):
                secondary(one, name, lambda n=name: one_gpu_sharded_line(wg, dev, n, flush, fp32_peak, fp64_peak))
        barrier(world)
        if rank == 0:
            eff = {}
            t1 = one.get(wname, {}).get("tflops")
            if t1:
                eff[wname] = value / (world * t1)
            td = one.get("shard16384d", {}).get("tflops")
            if td and "shard16384d" in extra:
                eff["shard16384d"] = extra["shard16384d"]["tflops"] / (world * td)
            extra["one_gpu_same_config"] = one
            extra["efficiency_same_config"] = eff
            extra["panels"] = secondary_value(lambda: panel_plan(wg, w, world))

    # Roofline of the dominant kernel, from the per-kernel events of the timed region.
    # Sharded: this rank's share of the product runs as several panel launches per
    # step, so achieved = the rank's FLOPs per step / the kernel's time per step.
    dom = max(prof.items(), key=lambda kv: kv[1][1]) if prof else ("?", (1, step_ms))
    dom_ms = dom[1][1] / max(dom[1][0], 1)
    rank_share = 1.0
    if w.get("sharded"):
        from wgblas_b200.shard import plan_rows

        offs = plan_rows(w["m"], world)
        rank_share = (offs[rank + 1] - offs[rank]) / w["m"]
    achieved = flops(w) * rank_share / (dom[1][1] / args.steps * 1e-3) / 1e12
    if dom[0].startswith("sgemm_tf32x3"):
        # A long sharded step can settle under the power cap: when the SM clock seen
        # during the timed region sat below its maximum, the step is held to the
        # sustained figure, else to the burst one.
        held = (w.get("sharded") and clocks.get("sm_mhz") and clocks.get("sm_max_mhz")
                and clocks["sm_mhz"] < 0.97 * clocks["sm_max_mhz"])
        key = "bf16_tflops_sustained" if held else "bf16_tflops"
        peak = peaks.get(key, FALLBACK_PEAKS[key]) * 0.5 / 3.0
        roof = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak, "traffic": None,
                "peak_basis": f"{peak_src} {key} x 0.5 (tf32 rate) / 3 products = 3xTF32 ceiling in fp32 FLOPs"}
    elif dom[0] == "dgemm_dmma":
        peak = fp64_peak
        roof = {"bound": "fp64-tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak if peak else None, "traffic": None,
                "peak_basis": "max of the DMMA-chain and DFMA-chain probes measured in this run"}
    else:
        peak = (fp64_peak if w["routine"] == "dgemm" else fp32_peak) or None
        roof = {"bound": "fp64-simt" if w["routine"] == "dgemm" else "fp32-simt", "achieved": achieved,
                "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak if peak else None, "traffic": None,
                "peak_basis": "FMA-chain probe measured in this run (no FP32/FP64 SIMT figure in MEASURED_PEAKS.json)"}
    traffic = NCU_TRAFFIC.get((wname, dom[0]))
    if traffic:
        roof["traffic"] = traffic[0] + traffic[1]
        roof["traffic_unit"] = "bytes per launch (DRAM read + write)"
        roof["traffic_source"] = f"ncu capture of this kernel and workload, {traffic[2]}"
    roof["kernel"] = dom[0]
    roof["kernel_ms"] = dom_ms
    roof["launches_per_step"] = dom[1][0] / args.steps
    roof["kernels"] = {k: {"launches": v[0], "avg_ms": v[1] / max(v[0], 1)} for k, v in prof.items()}

    if w.get("sharded") and world > 1:
        e2e = time_e2e_sharded(wg, dev, comm, w, short, args.warmup, world, rank)
    elif rank == 0 and not w.get("sharded"):
        e2e = time_e2e(wg, dev, w, short, args.warmup)
    else:
        e2e = None
    cb = None if (args.no_cpu_baseline or rank != 0 or world > 1) else cpu_baseline(w)
    if not args.no_extra and world == 1 and not w.get("sharded"):
        # Level-2 lines and the other bandwidth patterns, after every figure the
        # headline line needs has been taken.
        for kind in ("hbm_read", "hbm_scale"):  # the other patterns of bandwidth.js
            try:
                extra["probes"][f"{kind}_gbs"] = dev.probe_peak(kind)
            except Exception as e:  # noqa: BLE001 (a secondary line must not cost the JSON line)
                extra["probes"][f"{kind}_error"] = str(e)
        for dt in ("f32", "f64"):
            secondary(extra, f"cublas_{'d' if dt == 'f64' else 's'}gemm4096",
                      lambda d=dt: time_cublas(d, short, 3, flush, local))
        for routine in ("sgemv", "dgemv"):
            for trans in ("no-transpose", "transpose"):
                key = f"{routine}4096_{'N' if trans == 'no-transpose' else 'T'}"
                secondary(extra, key, lambda r=routine, t=trans: time_gemv(wg, dev, r, t, short, 3, flush))
                if hbm and "gbs" in extra[key]:
                    extra[key]["pct_of_hbm_copy"] = 100.0 * extra[key]["gbs"] / hbm
    barrier(world)
    if rank == 0:
        config = config_of(w, args.workload, world)
        line = {"metric": METRIC, "value": value, "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": step_ms_max, "higher_is_better": True,
                "scaling": "strong",
                "vs_baseline": None, "dtype": "f64" if w["routine"] == "dgemm" else "f32",
                "data": "synthetic (seeded mulberry32)", "config": config,
                "roofline": roof, "cpu_baseline": cb, "e2e": e2e, "parity": parity,
                "gpu_launches": launches_total,
                "clocks": clocks, "wall_s_timed_region": wall, "extra": extra,
                "summary": summary_of(value, parity, extra)}
        emit(line)
    if comm is not None:
        comm.destroy()
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    return 0


def secondary_value(fn):
    try:
        return fn()
    except Exception as e:  # noqa: BLE001
        return {"error": f"{type(e).__name__}: {e}"}


def summary_of(value, parity, extra):
    """Compact figures of the line, last in it so that a truncated tail still holds them."""
    out = {"value_tflops": round(value, 2), "parity_ok": None if parity is None else parity.get("ok")}
    for key in ("dgemm4096", "sgemm512", "ragged", "shard16384_1gpu", "shard16384d_1gpu", "shard16384d"):
        x = extra.get(key)
        if isinstance(x, dict) and "tflops" in x:
            out[f"{key}_tflops"] = round(x["tflops"], 3)
            if isinstance(x.get("parity"), dict):
                out[f"{key}_parity_ok"] = x["parity"].get("ok")
    if "efficiency_same_config" in extra:
        out["efficiency_same_config"] = {k: round(v, 4) for k, v in extra["efficiency_same_config"].items()}
    return out


if __name__ == "__main__":
    sys.exit(main())
