"""Per-thread pinned host staging buffers for the bytes-in/bytes-out codec API.

The ``Codec`` protocol moves Python ``bytes``; copying through pinned memory
lets the host<->device transfers run at full link speed with
``cudaMemcpyAsync``.  Each thread reuses its own buffer (grown by doubling),
and every bytes-API call synchronises its stream before returning, so a
buffer is never reused while a transfer that reads or writes it is in flight.
"""
from __future__ import annotations

import threading

import numpy as np
import torch

_tls = threading.local()


def pinned(nbytes: int, slot: str = "in") -> torch.Tensor:
    """A pinned uint8 host tensor of at least ``nbytes`` bytes (first ``nbytes`` returned)."""
    bufs = getattr(_tls, "bufs", None)
    if bufs is None:
        bufs = _tls.bufs = {}
    buf = bufs.get(slot)
    if buf is None or buf.numel() < nbytes:
        cap = 1 << max(12, (max(nbytes, 1) - 1).bit_length())
        buf = torch.empty(cap, dtype=torch.uint8, pin_memory=True)
        bufs[slot] = buf
    return buf[:nbytes]


def host_view(t: torch.Tensor) -> np.ndarray:
    """numpy view (no copy) of a CPU uint8 tensor."""
    return t.numpy()


def device() -> torch.device:
    return torch.device("cuda", torch.cuda.current_device())


def check_even(source_bytes: bytes) -> None:
    """Mirror torch.frombuffer's error for a bf16 buffer of odd byte length."""
    if len(source_bytes) % 2:
        raise ValueError(f"buffer length ({len(source_bytes)} bytes) after offset (0 bytes) "
                         f"must be a multiple of element size (2)")
