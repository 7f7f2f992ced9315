"""The dithered encoder divides its per-group absmax by half = (2^bits - 1) / 2 with
Markstein's correction instead of an IEEE division (ash-kv_b200/csrc/nbit_group.cuh).
This compiles the same three-step arithmetic in C with hardware fused multiply-add
and checks it against IEEE division for every finite float >= 1e-8, for each half."""
from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

SRC = Path(__file__).resolve().parent / "native" / "markstein_half.c"


def test_markstein_division_by_half_is_exact(tmp_path):
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    exe = tmp_path / "markstein_half"
    r = subprocess.run([cc, "-O2", "-ffp-contract=off", "-mfma", "-fno-math-errno", str(SRC), "-o", str(exe), "-lm"],
                       capture_output=True, text=True)
    if r.returncode != 0:
        pytest.skip("no FMA-capable C target: " + r.stderr[-200:])
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stdout
    assert out.stdout.count(" 0 of ") == 3, out.stdout
