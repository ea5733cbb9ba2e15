"""bench.py's command line on CPU: `--shape` times one sgemm of the given shape
(here through the reference arm, the oracle's FMA restatement) and labels the
line with it."""
from __future__ import annotations

import json
import os
import subprocess
import sys

from conftest import ROOT


def test_shape_option_on_the_reference_arm():
    r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--shape",
                        "96,64,40,1,0", "--steps", "1", "--warmup", "3"], cwd=ROOT, capture_output=True,
                       text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    assert line["config"]["workload"].startswith("shape sgemm 96x64x40 TN")
    assert (line["config"]["m"], line["config"]["n"], line["config"]["k"]) == (96, 64, 40)
    assert line["config"]["lda"] == 40 and line["config"]["ldb"] == 40 and line["config"]["ldc"] == 96
    assert line["value"] > 0 and line["unit"] == "TFLOP/s"
