"""The roofline report (wgblas_b200.roofline, the counterpart of the reference's
scripts/roofline.mjs over benchmarks/results-reader.mjs:504-584) on a recorded
bench line (tests/golden/bench_line_sample.json: a 1x B200 run of bench.py with
the routine and shape fields bench.py records for each row). CPU only."""
from __future__ import annotations

import copy
import json
import os

import pytest

from conftest import GOLDEN, load_golden

PEAKS = {"bf16_tflops": 1691.3}


@pytest.fixture(scope="module")
def rl(wg):
    from wgblas_b200 import roofline

    return roofline


@pytest.fixture()
def line():
    return load_golden("bench_line_sample.json")


def test_roofs_are_the_runs_own_probes(rl, line):
    roofs = rl.roofs_from(line, PEAKS)
    probes = line["extra"]["probes"]
    assert roofs.hbm_gbs == pytest.approx(probes["hbm_copy_gbs"])
    assert roofs.fp32_tflops == pytest.approx(1691.3 / 6)  # 3xTF32 ceiling above the FFMA probe
    assert roofs.fp64_tflops == pytest.approx(max(probes["fp64_dfma_tflops"], probes["fp64_dmma_tflops"]))
    no_tc = rl.roofs_from(line, None)
    assert no_tc.fp32_tflops == pytest.approx(probes["fp32_ffma_tflops"])
    assert rl.roofs_from({"extra": {}}, PEAKS) is None


def test_best_bandwidth_pattern_is_the_memory_roof(rl, line):
    line["extra"]["probes"]["hbm_read_gbs"] = line["extra"]["probes"]["hbm_copy_gbs"] * 1.05
    assert rl.roofs_from(line, PEAKS).hbm_gbs == pytest.approx(line["extra"]["probes"]["hbm_read_gbs"])


def test_reference_flop_and_byte_counts(rl):
    sh = {"m": 4096, "n": 4096, "k": 4096}
    g = rl.ROUTINES["sgemm"]
    assert g.flops(sh) == 2 * 4096**3 + 2 * 4096**2
    assert g.bytes(sh) == (3 * 4096**2 + 4096**2) * 4
    assert rl.ROUTINES["dgemm"].bytes(sh) == 2 * g.bytes(sh)
    assert rl.ROUTINES["ssyrk"].flops(sh) == 4096 * 4097 * 4096
    t = {"m": 4096, "n": 64, "aOrder": 4096}
    assert rl.ROUTINES["strsm"].flops(t) == 4096 * 64 * 4096
    assert rl.ROUTINES["strsm"].bytes(t) == (4096 * 4097 / 2 + 2 * 4096 * 64) * 4
    v = {"m": 4096, "n": 1024, "trans": "transpose"}
    assert rl.ROUTINES["sgemv"].flops(v) == 2 * 4096 * 1024
    assert rl.ROUTINES["sgemv"].bytes(v) == (4096 * 1024 + 4096 + 2 * 1024) * 4
    assert rl.ROUTINES["dgemv"].bytes(dict(v, trans="no-transpose")) == (4096 * 1024 + 1024 + 2 * 4096) * 8
    assert rl.ROUTINES["sgemv"].level == 2


def test_every_row_is_placed_with_its_bound(rl, line):
    points, skipped = rl.points_from(line)
    assert not skipped
    names = {p.name for p in points}
    assert {"headline", "dgemm4096", "ssymm4096", "strmm4096", "strsm4096_n64", "strsm4096_n4096"} <= names
    roofs = rl.roofs_from(line, PEAKS)
    by = {p.name: p for p in points}
    flops = rl.ROUTINES["sgemm"].flops({"m": 4096, "n": 4096, "k": 4096})
    assert by["headline"].tflops == pytest.approx(flops / (line["ms_per_step"] * 1e-3) / 1e12)
    assert by["strsm4096_n64"].ai < roofs.ridge("fp32") < by["headline"].ai
    # left of the ridge % of roof is GB/s over the memory roof, right of it FLOP/s over compute
    p = by["strsm4096_n64"]
    assert rl.pct_of_roof(p, roofs) == pytest.approx(100 * p.gbs / roofs.hbm_gbs)
    h = by["headline"]
    assert rl.pct_of_roof(h, roofs) == pytest.approx(100 * h.tflops / roofs.fp32_tflops)
    assert rl.attainable(p, roofs) == pytest.approx(p.ai * roofs.hbm_gbs / 1e3)
    assert not rl.above_roofs(points, roofs)


def test_rows_above_the_roof_are_flagged_not_dropped(rl, line):
    bad = copy.deepcopy(line)
    bad["extra"]["sgemm512"]["shape"] = {"m": 51200, "n": 512, "k": 512}  # a FLOP count 100x the work
    points, _ = rl.points_from(bad)
    over = rl.above_roofs(points, rl.roofs_from(bad, PEAKS))
    assert [p.name for p, _ in over] == ["sgemm512"]
    assert "above the measured roofs" in rl.report(bad, PEAKS)


def test_unplaceable_rows_are_listed(rl, line):
    bad = copy.deepcopy(line)
    del bad["extra"]["ragged"]["shape"]
    bad["extra"]["sgemm512"]["routine"] = "sgemv_experiment"
    bad["extra"]["dgemm4096"]["shape"] = {"m": 4096, "n": 4096}
    _, skipped = rl.points_from(bad)
    reasons = dict(skipped)
    assert reasons["ragged"] == "no size recorded"
    assert reasons["sgemm512"].startswith("not a roofline routine")
    assert reasons["dgemm4096"] == "missing size k"
    text = rl.report(bad, PEAKS, verbose=True)
    assert "rows not placed" in text and "ragged: no size recorded" in text


def test_multi_gpu_and_reference_lines(rl, line, tmp_path, capsys):
    multi = dict(copy.deepcopy(line), n_gpus=8)
    assert all(p.name != "headline" for p in rl.points_from(multi)[0])
    path = tmp_path / "runs.json"
    ref = {"impl": "reference", "metric": "x", "value": 1.0}
    path.write_text(json.dumps(line) + "\n" + json.dumps(ref) + "\n")
    peaks = tmp_path / "peaks.json"
    peaks.write_text(json.dumps(PEAKS))
    assert rl.main([str(path), "--peaks", str(peaks)]) == 0
    out = capsys.readouterr().out
    assert out.count("roofs:") == 1 and "strsm4096_n64" in out
    assert os.path.exists(os.path.join(GOLDEN, "bench_line_sample.json"))
