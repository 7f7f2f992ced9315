"""The reference arm's host-core harness (oracle/reference_shim.py).

The bench's reference arm times the reference's own ``DitheredNBitCodec`` with
its CUDA calls redirected to the CPU.  This checks, in a child interpreter
(the reference is imported under its own package name ``ashkv``), that the
harness runs the reference code faithfully: with the fixture's uniforms
injected it reproduces the reference-generated blobs and decodes byte for
byte, and with its own CPU generator it round-trips config-2 data.
"""
from __future__ import annotations

import subprocess
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(REPO))

from oracle import reference_copy  # noqa: E402

CHILD = r'''
import sys
sys.path.insert(0, sys.argv[1])
import numpy as np, torch
from oracle import reference_shim
Codec = reference_shim.load_reference_codecs()
z = np.load(sys.argv[2])
checked = 0
for ci in range(int(z["nbit_n_cases"])):
    bits, hidden, is_int2, n, trailing = (int(v) for v in z[f"nbit_{ci}_meta"])
    if is_int2 or n == 0:
        continue
    codec = Codec(hidden_dim=hidden, group_size=32, sigma=float(z[f"nbit_{ci}_sigma"]), bits=bits)
    U = torch.from_numpy(z[f"nbit_{ci}_u"]).view(n // hidden, hidden // 32, 32)
    with reference_shim.CpuShim(U):
        blob = codec.encode(z[f"nbit_{ci}_src"].tobytes())
        dec = codec.decode(blob)
    assert blob == z[f"nbit_{ci}_blob"].tobytes(), ci
    assert dec == z[f"nbit_{ci}_decoded"].tobytes(), ci
    checked += 1
assert checked >= 5, checked
rate, info = reference_shim.reference_nbit_rate([np.zeros(16 * 8 * 128 * 4, np.uint16).tobytes()], 0.0, 2)
assert rate > 0 and info["calls"] == 1
print("OK", checked)
'''


@pytest.mark.skipif(not reference_copy.available(), reason="no copy of the reference in oracle/_ref")
def test_reference_shim_reproduces_reference_fixtures():
    r = subprocess.run([sys.executable, "-c", CHILD, str(REPO), str(REPO / "tests" / "golden" / "nbit.npz")],
                       capture_output=True, text=True, timeout=600, cwd=str(REPO))
    assert r.returncode == 0, r.stdout + r.stderr
    assert r.stdout.startswith("OK")
