"""The reference's own test files, run unchanged against this package on a GPU.

``oracle/reference_copy.py`` copies the reference package into
``oracle/_ref/ashkv`` (git-ignored; it travels with the working tree to the GPU
machine).  Each file below is run by pytest in a child process with
``--import-mode=importlib`` and this repository's ``ash-kv_b200`` first on
``PYTHONPATH``, so every ``import ashkv`` in the reference's tests resolves to
this package.  The test files are the checker; nothing of the reference's
package is imported.

Two tests of ``test_ashkv_local.py`` are deselected: ``test_telemetry_byte_math``
and ``test_telemetry_flush_debounce`` replace the hooks' Triton kernel getter
with a mock so that the reference hook can run on CPU tensors
(``ashkv/tests/test_ashkv_local.py:15-49, 110-160``).  This package has no CPU
path (its hooks launch CUDA kernels on the pools' own device), so the mock
cannot stand in for anything here; the same stats arithmetic is covered by
``tests/test_gpu_adapters.py`` on real CUDA pools.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest

from oracle import reference_copy

REPO = Path(__file__).resolve().parents[1]

SUITES = {
    "test_runtime.py": None,
    "test_contracts.py": None,
    "test_migrate_fault_injection.py": None,
    "test_ashkv_gpu.py": None,
    "test_ashkv_local.py": "not test_telemetry_byte_math and not test_telemetry_flush_debounce",
}


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(SUITES))
def test_reference_suite(name, tmp_path):
    if not reference_copy.available():
        pytest.skip("no copy of the reference package in oracle/_ref (made by oracle/reference_copy.py)")
    path = reference_copy.REF_PACKAGE / "tests" / name
    cmd = [sys.executable, "-m", "pytest", "-q", "-p", "no:cacheprovider", "--import-mode=importlib",
           "-c", os.devnull, "--rootdir", str(tmp_path), str(path)]
    if SUITES[name]:
        cmd += ["-k", SUITES[name]]
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join([str(REPO / "ash-kv_b200"), str(REPO)] +
                                        ([env["PYTHONPATH"]] if env.get("PYTHONPATH") else []))
    r = subprocess.run(cmd, cwd=tmp_path, env=env, capture_output=True, text=True, timeout=900)
    tail = (r.stdout + r.stderr)[-4000:]
    assert r.returncode == 0, f"reference suite {name} failed:\n{tail}"
    assert " passed" in r.stdout, tail
    # the same interpreter set-up resolves ``ashkv`` to this package, not to the copy
    who = subprocess.run([sys.executable, "-c", "import ashkv; print(ashkv.__file__)"], cwd=tmp_path, env=env,
                         capture_output=True, text=True, timeout=300)
    assert Path(who.stdout.strip()).resolve().is_relative_to(REPO / "ash-kv_b200"), who.stdout + who.stderr
