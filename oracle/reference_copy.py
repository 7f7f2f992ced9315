"""Copy of the reference package for checks that run the reference itself — TEST INFRASTRUCTURE ONLY.

The reference ASH-KV is a pure Python/Triton package.  Its two Triton INT8
kernels, its SGLang hooks and its simulator only run on a CUDA GPU, so the
fixtures that pin this library's bf16 INT8 path, hook slot bytes and
attention saliency to the reference's own outputs are generated on a B200
(``tests/golden/make_golden_gpu.py``), and the reference's own test files are
run against this package there (``tests/test_gpu_reference_suite.py``).  The
GPU machine sees only this working tree, so ``copy_reference()`` copies the
reference's ``ashkv/`` package into ``oracle/_ref/ashkv`` (git-ignored, never
committed, never imported by the product).

Source location: ``$ASHKV_REFERENCE`` if set, else the read-only mount
``/root/reference`` of the build container.  Nothing happens when neither
exists (on the GPU machine the copy made in the build container is used).
"""
from __future__ import annotations

import os
import shutil
from pathlib import Path
from typing import Optional

ORACLE_DIR = Path(__file__).resolve().parent
REF_DIR = ORACLE_DIR / "_ref"
REF_PACKAGE = REF_DIR / "ashkv"
DEFAULT_SOURCE = Path("/root/reference")


def reference_source() -> Optional[Path]:
    env = os.environ.get("ASHKV_REFERENCE")
    for cand in ([Path(env)] if env else []) + [DEFAULT_SOURCE]:
        if (cand / "ashkv" / "__init__.py").is_file():
            return cand
    return None


def copy_reference(force: bool = False) -> Optional[Path]:
    """Copy ``<reference>/ashkv`` to ``oracle/_ref/ashkv``; returns the copy (or None if no source)."""
    src = reference_source()
    if src is None:
        return REF_PACKAGE if REF_PACKAGE.is_dir() else None
    if REF_PACKAGE.is_dir() and not force:
        return REF_PACKAGE
    REF_DIR.mkdir(parents=True, exist_ok=True)
    tmp = REF_DIR / "ashkv.tmp"
    if tmp.exists():
        shutil.rmtree(tmp)
    shutil.copytree(src / "ashkv", tmp, ignore=shutil.ignore_patterns("__pycache__", "*.pyc"))
    if REF_PACKAGE.exists():
        shutil.rmtree(REF_PACKAGE)
    os.replace(tmp, REF_PACKAGE)
    return REF_PACKAGE


def available() -> bool:
    return (REF_PACKAGE / "__init__.py").is_file()


if __name__ == "__main__":
    print(copy_reference(force=True))
