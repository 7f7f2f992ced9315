"""The reference's Triton INT8 kernel run live on the B200 as the checker.

The committed B200 fixtures pin the INT8 path on a few thousand rows.  Here the
reference's own ``_int8_encode_kernel`` (``ashkv/codecs/int8.py:50-81``, from the
copy in ``oracle/_ref``) runs in a child process on the same GPU over every
quotient a row can form in one binade of absmax values — for every bf16 absmax
in [1, 2), rows holding every bf16 value of magnitude up to it — and this
library's kernel, through the C ABI, must return the same codes and scales
bit for bit, with bf16 and fp16 scale buffers (the quotient's rounding is
invariant under power-of-two scaling of both operands, so one binade covers
the whole range below 2^126).
"""
from __future__ import annotations

import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import reference_copy

from ashkv.codecs import int8 as int8_mod

pytestmark = pytest.mark.gpu

REPO = Path(__file__).resolve().parents[1]

CHILD = r'''
import sys
import numpy as np
import torch
sys.path.insert(0, sys.argv[1])
from ashkv.codecs.int8 import _get_kernels  # the reference's Triton kernels
enc, _ = _get_kernels()
z = np.load(sys.argv[2])
out = {}
for key in z.files:
    bits = z[key]
    n, L = bits.shape
    src = torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).cuda()
    for sname, sdt in (("bf16", torch.bfloat16), ("fp16", torch.float16)):
        codes = torch.empty((n, L), dtype=torch.int8, device="cuda")
        scales = torch.empty((n,), dtype=sdt, device="cuda")
        enc[(n,)](src, codes, scales, n, L)
        torch.cuda.synchronize()
        out[f"{key}_{sname}_codes"] = codes.cpu().numpy()
        out[f"{key}_{sname}_scales"] = scales.cpu().view(torch.int16).numpy()
np.savez(sys.argv[3], **out)
print("OK")
'''


def binade_rows(L: int) -> np.ndarray:
    rows = []
    for a in list(range(0x3F80, 0x4000)) + [0x0001, 0x0080, 0x3300, 0x7F7F]:
        mags = np.arange(0, a + 1, dtype=np.uint32)
        vals = np.concatenate([mags, mags | 0x8000]).astype(np.uint16)
        vals = np.concatenate([vals, np.zeros((-len(vals)) % (L - 1), np.uint16)]).reshape(-1, L - 1)
        rows.append(np.concatenate([np.full((len(vals), 1), a, np.uint16), vals], axis=1))
    return np.concatenate(rows)


@pytest.mark.skipif(not reference_copy.available(), reason="no copy of the reference in oracle/_ref")
def test_int8_every_quotient_of_a_binade_equals_reference_triton(cuda, tmp_path):
    inputs = {f"L{L}": binade_rows(L) for L in (128, 1024)}
    np.savez(tmp_path / "in.npz", **inputs)
    r = subprocess.run([sys.executable, "-c", CHILD, str(reference_copy.REF_DIR), str(tmp_path / "in.npz"),
                        str(tmp_path / "ref.npz")], capture_output=True, text=True, timeout=900, cwd=str(tmp_path))
    assert r.returncode == 0, r.stdout + r.stderr
    ref = np.load(tmp_path / "ref.npz")
    for key, bits in inputs.items():
        n, L = bits.shape
        x = torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).to(cuda)
        for sname, sdt in (("bf16", torch.bfloat16), ("fp16", torch.float16)):
            codes, scales = int8_mod.encode_rows(x, scale_dtype=sdt)
            got_c = codes.cpu().numpy()
            want_c = ref[f"{key}_{sname}_codes"]
            bad = np.argwhere(got_c != want_c)
            assert bad.size == 0, (key, sname, len(bad), bad[:5].tolist())
            assert np.array_equal(scales.cpu().view(torch.int16).numpy(), ref[f"{key}_{sname}_scales"]), (key, sname)
