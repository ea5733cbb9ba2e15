"""Repository hygiene (CPU): committed code and profile summaries never reach into
the working folder, and every profile summary names the command that made it."""
from __future__ import annotations

import os
import subprocess

from conftest import ROOT

WORK = "_" + "work"  # the working folder's name, spelled so this file does not contain it


def _tracked():
    out = subprocess.run(["git", "ls-files"], cwd=ROOT, capture_output=True, text=True)
    if out.returncode != 0:  # not a git checkout (a copied tree): walk it instead
        files = []
        for d, dirs, names in os.walk(ROOT):
            dirs[:] = [x for x in dirs if not x.startswith((".", WORK, "_build", "gpurun_out", "baseline"))]
            files += [os.path.relpath(os.path.join(d, n), ROOT) for n in names]
        return files
    return out.stdout.split()


def test_nothing_committed_uses_the_working_folder():
    for rel in _tracked():
        if rel.endswith((".py", ".cu", ".cuh", ".h", ".c", ".cpp", ".sh", "Makefile")):
            text = open(os.path.join(ROOT, rel), errors="replace").read()
            assert WORK + "/" not in text, rel


def test_profile_summaries_name_their_command():
    pdir = os.path.join(ROOT, "profiles")
    names = [n for n in os.listdir(pdir) if n.endswith((".md", ".txt"))]
    assert names
    for n in names:
        text = open(os.path.join(pdir, n)).read()
        assert WORK + "/" not in text, n
        assert "python bench.py" in text or "python -m pytest" in text or "python -m wgblas_b200" in text, n
