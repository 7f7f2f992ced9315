"""Run the reference's own dithered N-bit codec on the host cores — TEST AND CPU-BASELINE INFRASTRUCTURE ONLY.

The reference's ``DitheredNBitCodec`` (ashkv/codecs/nbit_dithered.py:43-167)
is PyTorch code that moves every tensor to CUDA (``.cuda()``,
``torch.empty(..., device="cuda")``) and draws its dither from a generator on
that device.  ``CpuShim`` runs those unchanged function bodies on the CPU:
``Tensor.cuda`` becomes the identity and CUDA ``torch.empty`` allocates on the
CPU, so the generator the codec creates (``torch.Generator(device=arr.device)``)
is a CPU generator with the codec's own seed.  Optionally ``torch.rand``
returns an injected uniform tensor instead (``CpuShim(U)``), which is how the
parity fixtures fix the dither.

``reference_nbit_rate`` times that code (encode + decode through its bytes
API, all host threads via ``torch.set_num_threads``) on chunks of the
INT4 dithered workload; the bench's reference arm reports it.  The reference
package is the copy made by ``oracle/reference_copy.py`` in ``oracle/_ref``;
it is imported under its own name ``ashkv``, so this runs in a process that
has not imported this library's ``ashkv`` package.
"""
from __future__ import annotations

import os
import sys
import time
from typing import Optional

from oracle import reference_copy


class CpuShim:
    """Context manager: CUDA calls of the reference codec land on the CPU."""

    def __init__(self, U=None):
        import torch
        self.torch = torch
        self.U = U

    def __enter__(self):
        torch = self.torch
        self._cuda = torch.Tensor.cuda
        self._rand = torch.rand
        self._empty = torch.empty
        shim = self

        def cuda(self_t, *a, **k):
            return self_t

        def rand(*size, generator=None, device=None, dtype=None, **kw):
            if shim.U is None:
                return shim._rand(*size, generator=generator, dtype=dtype, **kw)
            if len(size) == 1 and isinstance(size[0], (tuple, list, torch.Size)):
                size = tuple(size[0])
            assert tuple(shim.U.shape) == tuple(size), (shim.U.shape, size)
            return shim.U.clone()

        def empty(*size, device=None, **kw):
            return shim._empty(*size, **kw)

        torch.Tensor.cuda = cuda
        torch.rand = rand
        torch.empty = empty
        return self

    def __exit__(self, *exc):
        self.torch.Tensor.cuda = self._cuda
        self.torch.rand = self._rand
        self.torch.empty = self._empty
        return False


def load_reference_codecs():
    """Import the reference package from ``oracle/_ref``; None when the copy is absent."""
    if not reference_copy.available():
        return None
    mod = sys.modules.get("ashkv")
    ref_root = str(reference_copy.REF_DIR)
    if mod is not None and not str(getattr(mod, "__file__", "")).startswith(ref_root):
        raise RuntimeError("this library's ashkv package is already imported; the reference "
                           "codec must be timed in a process of its own")
    if ref_root not in sys.path:
        sys.path.insert(0, ref_root)
    from ashkv.codecs.nbit_dithered import DitheredNBitCodec  # the reference's class
    return DitheredNBitCodec


def reference_nbit_rate(chunks, budget_s: float, threads: Optional[int] = None,
                        bits: int = 4, sigma: float = 3.0) -> Optional[tuple[float, dict]]:
    """bf16 GB/s (bytes of bf16 input carried through encode and decode) of the
    reference codec over ``chunks`` (bf16 byte strings).

    Runs chunks round-robin until ``budget_s`` has passed; returns (GB/s, info)
    or None when the reference copy is absent.
    """
    import torch
    cls = load_reference_codecs()
    if cls is None:
        return None
    threads = threads or os.cpu_count() or 1
    torch.set_num_threads(threads)
    codec = cls(hidden_dim=128, group_size=32, sigma=sigma, bits=bits)
    done = calls = 0
    t0 = time.perf_counter()
    with CpuShim():
        while True:
            src = chunks[calls % len(chunks)]
            blob = codec.encode(src)
            out = codec.decode(blob)
            assert len(out) == len(src)
            done += len(src)
            calls += 1
            if time.perf_counter() - t0 >= budget_s:
                break
    dt = time.perf_counter() - t0
    return done / dt / 1e9, {"bytes": done, "calls": calls, "seconds": round(dt, 3), "threads": threads}
