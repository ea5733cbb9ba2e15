"""Roofline report over this library's benchmark results.

The B200 counterpart of the reference's maintainer tooling: scripts/roofline.mjs
(the table and its two checks) over benchmarks/results-reader.mjs:504-584
(readRoofline), with each routine's FLOP and byte counts as the reference's
benchmarks count them (benchmarks/<routine>/wgblas/<routine>.js, cited per
routine below).

Input: JSON lines as ``bench.py`` prints them (one line per run; a file may hold
several). The headline's ``config`` and every secondary row in
``extra`` carry ``routine``, ``shape`` and ``ms_per_step``; rows without them
are listed as not placed, as the reference lists rows it cannot place.

Roofs are measured, never typed in. The memory roof is the best of the HBM
probes the same run recorded (copy, read-only, in-place scale: the patterns of
benchmarks/roofline/wgblas/bandwidth.js). A B200 has several compute roofs
where the reference's GPU has one FMA roof: fp32 routines run on the 3xTF32
tensor-core path, so their roof is the faster of the FFMA-chain probe and the
3xTF32 ceiling (the measured dense bf16 rate x 1/2 for TF32 x 1/3 for three
products); fp64 routines take the faster of the DFMA and DMMA probes.

    python -m wgblas_b200.roofline BENCH.json [more.json ...] [--peaks MEASURED_PEAKS.json] [-v]
"""
from __future__ import annotations

import argparse
import json
import sys
from dataclasses import dataclass
from typing import Callable


@dataclass(frozen=True)
class Routine:
    level: int
    precision: str  # "fp32" or "fp64": which compute roof applies
    flops: Callable[[dict], float]
    bytes: Callable[[dict], float]
    source: str


def _gemm(elt):
    return (lambda p: 2.0 * p["m"] * p["n"] * p["k"] + 2.0 * p["m"] * p["n"],
            lambda p: (p["m"] * p["k"] + p["k"] * p["n"] + 2.0 * p["m"] * p["n"]) * elt)


def _gemmtr(elt):
    return (lambda p: float(p["n"]) * (p["n"] + 1) * p["k"],
            lambda p: (p["m"] * p["k"] + p["k"] * p["n"] + 1.0 * p["m"] * p["n"]) * elt)


def _syrk(elt):
    return (lambda p: float(p["n"]) * (p["n"] + 1) * p["k"], lambda p: (p["n"] * p["k"] + 1.0 * p["n"] * p["n"]) * elt)


def _syr2k(elt):
    return (lambda p: 2.0 * p["n"] * (p["n"] + 1) * p["k"],
            lambda p: (2.0 * p["n"] * p["k"] + 1.0 * p["n"] * p["n"]) * elt)


def _symm(elt):
    return (lambda p: 2.0 * p["m"] * p["n"] * p["aOrder"] + 2.0 * p["m"] * p["n"],
            lambda p: (3.0 * p["aOrder"] * p["aOrder"] + 3.0 * p["m"] * p["n"]) * elt)


def _trmm(elt):
    return (lambda p: 2.0 * p["m"] * p["n"] * p["aOrder"] + 1.0 * p["m"] * p["n"],
            lambda p: (3.0 * p["aOrder"] * p["aOrder"] + 5.0 * p["m"] * p["n"]) * elt)


def _trsm(elt):
    return (lambda p: float(p["m"]) * p["n"] * p["aOrder"],
            lambda p: (p["aOrder"] * (p["aOrder"] + 1) / 2.0 + 2.0 * p["m"] * p["n"]) * elt)


def _gemv(elt):
    def lens(p):
        no_t = p.get("trans", "no-transpose") == "no-transpose"
        return (p["n"], p["m"]) if no_t else (p["m"], p["n"])

    return (lambda p: 2.0 * p["m"] * p["n"],
            lambda p: (1.0 * p["m"] * p["n"] + lens(p)[0] + 2.0 * lens(p)[1]) * elt)


def _routine(level, precision, pair, source):
    return Routine(level, precision, pair[0], pair[1], source)


ROUTINES = {
    "sgemm": _routine(3, "fp32", _gemm(4), "benchmarks/sgemm/wgblas/sgemm.js:73-75"),
    "dgemm": _routine(3, "fp64", _gemm(8), "benchmarks/dgemm/wgblas/dgemm.js:72-74"),
    "sgemmtr": _routine(3, "fp32", _gemmtr(4), "benchmarks/sgemmtr/wgblas/sgemmtr.js:56-58"),
    "dgemmtr": _routine(3, "fp64", _gemmtr(8), "benchmarks/dgemmtr/wgblas/dgemmtr.js:55-57"),
    "ssyrk": _routine(3, "fp32", _syrk(4), "benchmarks/ssyrk/wgblas/ssyrk.js:58-60"),
    "dsyrk": _routine(3, "fp64", _syrk(8), "benchmarks/dsyrk/wgblas/dsyrk.js:56-58"),
    "ssyr2k": _routine(3, "fp32", _syr2k(4), "benchmarks/ssyr2k/wgblas/ssyr2k.js:62-64"),
    "dsyr2k": _routine(3, "fp64", _syr2k(8), "benchmarks/dsyr2k/wgblas/dsyr2k.js:55-57"),
    "ssymm": _routine(3, "fp32", _symm(4), "benchmarks/ssymm/wgblas/ssymm.js:55-58"),
    "dsymm": _routine(3, "fp64", _symm(8), "benchmarks/dsymm/wgblas/dsymm.js:55-58"),
    "strmm": _routine(3, "fp32", _trmm(4), "benchmarks/strmm/wgblas/strmm.js:51-55"),
    "dtrmm": _routine(3, "fp64", _trmm(8), "benchmarks/dtrmm/wgblas/dtrmm.js:50-54"),
    "strsm": _routine(3, "fp32", _trsm(4), "benchmarks/strsm/wgblas/strsm.js:55-58"),
    "sgemv": _routine(2, "fp32", _gemv(4), "assets/routines/routine_params.json (flops), "
                      "benchmarks/sgemv/wgblas/sgemv.js:49 (bytes)"),
    "dgemv": _routine(2, "fp64", _gemv(8), "benchmarks/dgemv/wgblas/dgemv.js:49"),
}


@dataclass(frozen=True)
class Roofs:
    fp32_tflops: float
    fp64_tflops: float
    hbm_gbs: float
    source: str

    def compute(self, precision: str) -> float:
        return self.fp32_tflops if precision == "fp32" else self.fp64_tflops

    def ridge(self, precision: str) -> float:
        """FLOP per byte where the sloped memory roof meets the compute roof."""
        return self.compute(precision) * 1e12 / (self.hbm_gbs * 1e9)


def roofs_from(line: dict, peaks: dict | None = None) -> Roofs | None:
    """The roofs of one bench run: its own probes, plus the 3xTF32 ceiling from the
    measured bf16 rate. None when the run recorded no probes (no measured roofs,
    as scripts/roofline.mjs skips a GPU without probe results)."""
    probes = (line.get("extra") or {}).get("probes")
    if not probes:
        return None
    hbm = max(v for k, v in probes.items() if k.startswith("hbm") and isinstance(v, (int, float)))
    fp32 = float(probes.get("fp32_ffma_tflops", 0.0))
    parts = ["probes of the same run"]
    bf16 = (peaks or {}).get("bf16_tflops")
    if bf16:
        fp32 = max(fp32, float(bf16) * 0.5 / 3.0)
        parts.append("3xTF32 ceiling = measured bf16 dense x 1/2 x 1/3")
    fp64 = max(float(probes.get("fp64_dfma_tflops", 0.0)), float(probes.get("fp64_dmma_tflops", 0.0)))
    return Roofs(fp32, fp64, float(hbm), "; ".join(parts))


@dataclass
class Point:
    name: str
    routine: str
    level: int
    precision: str
    size: str
    flops: float
    bytes: float
    ms: float

    @property
    def ai(self) -> float:
        return self.flops / self.bytes if self.bytes else float("inf")

    @property
    def tflops(self) -> float:
        return self.flops / (self.ms * 1e-3) / 1e12

    @property
    def gbs(self) -> float:
        return self.bytes / (self.ms * 1e-3) / 1e9


def _size_label(shape: dict) -> str:
    keys = [k for k in ("m", "n", "k", "aOrder") if k in shape]
    return "x".join(str(shape[k]) for k in keys)


def _point(name: str, row: dict):
    """A Point, or the reason the row cannot be placed."""
    routine = row.get("routine")
    if routine is None:
        return "no routine recorded"
    r = ROUTINES.get(routine)
    if r is None:
        return f"not a roofline routine ({routine})"
    shape = row.get("shape")
    ms = row.get("ms_per_step")
    if not shape:
        return "no size recorded"
    if not ms or ms <= 0:
        return "no time recorded"
    try:
        fl, by = r.flops(shape), r.bytes(shape)
    except KeyError as e:
        return f"missing size {e.args[0]}"
    return Point(name, routine, r.level, r.precision, _size_label(shape), fl, by, float(ms))


def points_from(line: dict):
    """(points, skipped) of one bench line: the headline (for a single-GPU line) and
    every secondary row in ``extra``."""
    points, skipped = [], []
    rows = []
    cfg = line.get("config") or {}
    if line.get("n_gpus", 1) == 1 and line.get("impl", "ours") == "ours":
        rows.append(("headline", {"routine": cfg.get("routine"), "shape": cfg.get("shape"),
                                  "ms_per_step": line.get("ms_per_step")}))
    for name, row in (line.get("extra") or {}).items():
        if name == "probes" or not isinstance(row, dict):
            continue
        rows.append((name, row))
    for name, row in rows:
        p = _point(name, row)
        if isinstance(p, Point):
            points.append(p)
        else:
            skipped.append((name, p))
    return points, skipped


def attainable(p: Point, roofs: Roofs) -> float:
    """TFLOP/s the roofline allows at the point's intensity."""
    return min(roofs.compute(p.precision), p.ai * roofs.hbm_gbs * 1e9 / 1e12)


def pct_of_roof(p: Point, roofs: Roofs) -> float:
    """results-reader.mjs:549-556: left of the ridge, GB/s over the memory roof;
    right of it, FLOP/s over the compute roof."""
    if p.ai < roofs.ridge(p.precision):
        return 100.0 * p.gbs / roofs.hbm_gbs if roofs.hbm_gbs else 0.0
    peak = roofs.compute(p.precision)
    return 100.0 * p.tflops / peak if peak else 0.0


def above_roofs(points, roofs: Roofs):
    """Rows above the measured roofs, largest overshoot first (kept, never dropped:
    either the probe undershot or the row's FLOP or byte count is wrong)."""
    out = []
    for p in points:
        ratio = max(p.tflops / roofs.compute(p.precision), p.gbs / roofs.hbm_gbs)
        if ratio > 1.0:
            out.append((p, ratio))
    return sorted(out, key=lambda t: -t[1])


def report(line: dict, peaks: dict | None = None, verbose: bool = False) -> str:
    roofs = roofs_from(line, peaks)
    label = (line.get("config") or {}).get("workload", "run")
    if roofs is None:
        return f"{label}: skipped, no measured roofs (the run recorded no probes)\n"
    points, skipped = points_from(line)
    out = ["=" * 100,
           f"{label}",
           f"roofs: fp32 {roofs.fp32_tflops:.1f} TFLOP/s, fp64 {roofs.fp64_tflops:.1f} TFLOP/s, "
           f"HBM {roofs.hbm_gbs:.0f} GB/s ({roofs.source})",
           f"ridge points: fp32 {roofs.ridge('fp32'):.1f} FLOP/byte, fp64 {roofs.ridge('fp64'):.1f} FLOP/byte",
           "=" * 100]
    head = (f"{'row':<18}{'routine':<9}{'lvl':>4}{'size':>21}{'FLOP/B':>9}{'TFLOP/s':>10}{'GB/s':>9}"
            f"{'roof':>9}{'% roof':>8}  bound")
    out.append(head)
    out.append("-" * len(head))
    for p in sorted(points, key=lambda q: (q.level, q.routine, q.name)):
        bound = "compute" if p.ai >= roofs.ridge(p.precision) else "memory"
        out.append(f"{p.name:<18}{p.routine:<9}{p.level:>4}{p.size:>21}{p.ai:>9.1f}{p.tflops:>10.1f}"
                   f"{p.gbs:>9.0f}{attainable(p, roofs):>9.1f}{pct_of_roof(p, roofs):>7.0f}%  {bound}")
    over = above_roofs(points, roofs)
    if over:
        out.append(f"\n  {len(over)} row(s) above the measured roofs (kept):")
        for p, ratio in over[:8]:
            out.append(f"    {p.name:<18} {p.tflops:9.1f} TFLOP/s {p.gbs:8.0f} GB/s  {ratio:.2f}x roof")
    if skipped:
        out.append("\n  rows not placed:")
        counts = {}
        for _, why in skipped:
            counts[why] = counts.get(why, 0) + 1
        for why, n in sorted(counts.items(), key=lambda t: -t[1]):
            out.append(f"    {n:5d}  {why}")
        if verbose:
            for name, why in skipped:
                out.append(f"      {name}: {why}")
    return "\n".join(out) + "\n"


def read_lines(path: str):
    """The JSON objects of a file holding one bench line per line (or one JSON document)."""
    with open(path) as fh:
        text = fh.read().strip()
    if not text:
        return []
    try:
        doc = json.loads(text)
        return doc if isinstance(doc, list) else [doc]
    except json.JSONDecodeError:
        return [json.loads(ln) for ln in text.splitlines() if ln.strip().startswith("{")]


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="Roofline table of bench.py results.")
    ap.add_argument("results", nargs="+", help="files of bench.py JSON lines")
    ap.add_argument("--peaks", help="measured peaks JSON (bf16_tflops gives the 3xTF32 ceiling)")
    ap.add_argument("-v", "--verbose", action="store_true", help="also list every row not placed")
    a = ap.parse_args(argv)
    peaks = None
    if a.peaks:
        with open(a.peaks) as fh:
            peaks = json.load(fh)
    status = 0
    for path in a.results:
        lines = read_lines(path)
        if not lines:
            print(f"{path}: no results", file=sys.stderr)
            status = 1
        for line in lines:
            if line.get("impl") == "reference" or "unavailable" in line:
                continue
            sys.stdout.write(report(line, peaks, a.verbose))
    return status


if __name__ == "__main__":
    sys.exit(main())
