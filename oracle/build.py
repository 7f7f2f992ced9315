"""Build recipe for the oracle's C restatement — TEST INFRASTRUCTURE ONLY.

Compiles oracle/codec_oracle.c with gcc into oracle/_build/libcodec_oracle.so.
``-ffp-contract=off`` keeps every float operation a separate IEEE-754
operation (no fused multiply-add), which is how the reference's PyTorch code
evaluates on the host.
"""
from __future__ import annotations

import os
import shutil
import subprocess
from pathlib import Path

ORACLE_DIR = Path(__file__).resolve().parent
SRC = ORACLE_DIR / "codec_oracle.c"
LIB = ORACLE_DIR / "_build" / "libcodec_oracle.so"


def build(force: bool = False) -> Path:
    if not force and LIB.exists() and LIB.stat().st_mtime >= SRC.stat().st_mtime:
        return LIB
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        raise RuntimeError("gcc not found; the oracle cannot be built")
    LIB.parent.mkdir(parents=True, exist_ok=True)
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [cc, "-O2", "-std=c11", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-shared",
           str(SRC), "-o", str(tmp), "-lm"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"oracle build failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force=True))
