"""bench.py's DRAM traffic figures are the ones of the ncu captures summarised
in profiles/ (the summary files are the record; the bench reports them as the
roofline's `traffic`). CPU only."""
from __future__ import annotations

import importlib.util
import os
import re

from conftest import ROOT


def test_traffic_matches_the_profile_summaries():
    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(ROOT, "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    assert bench.NCU_TRAFFIC
    for (workload, kernel), (read, write, source) in bench.NCU_TRAFFIC.items():
        assert workload in bench.WORKLOADS
        with open(os.path.join(ROOT, source)) as fh:
            text = fh.read()
        m = re.search(r"dram__bytes_read\.sum / dram__bytes_write\.sum \| ([0-9.]+) MB / ([0-9.]+) MB", text)
        assert m, source
        assert (float(m.group(1)) * 1e6, float(m.group(2)) * 1e6) == (read, write)
        assert kernel.split("_")[0] in text
