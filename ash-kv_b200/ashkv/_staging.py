"""Per-thread pinned host staging buffers for the bytes-in/bytes-out codec API.

The ``Codec`` protocol moves Python ``bytes``; copying through pinned memory
lets the host<->device transfers run at full link speed with
``cudaMemcpyAsync``.  Each thread reuses its own buffer (grown by doubling),
and every bytes-API call synchronises its stream before returning, so a
buffer is never reused while a transfer that reads or writes it is in flight.
"""
from __future__ import annotations

import ctypes
import os
import threading
from concurrent.futures import ThreadPoolExecutor

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


# ---------------------------------------------------------------- parallel host copies
_CHUNK = 8 << 20          # split copies above this size across threads
_POOL: ThreadPoolExecutor | None = None
_POOL_LOCK = threading.Lock()

_new_bytes = ctypes.pythonapi.PyBytes_FromStringAndSize
_new_bytes.restype = ctypes.py_object
_new_bytes.argtypes = [ctypes.c_void_p, ctypes.c_ssize_t]
_bytes_ptr = ctypes.pythonapi.PyBytes_AsString
_bytes_ptr.restype = ctypes.c_void_p
_bytes_ptr.argtypes = [ctypes.py_object]


def _pool() -> ThreadPoolExecutor:
    global _POOL
    if _POOL is None:
        with _POOL_LOCK:
            if _POOL is None:
                _POOL = ThreadPoolExecutor(max_workers=min(16, os.cpu_count() or 1),
                                           thread_name_prefix="ashkv-memcpy")
    return _POOL


def memcpy(dst: int, src: int, n: int) -> None:
    """Host memcpy of n bytes; large copies are split over a thread pool
    (ctypes.memmove releases the GIL)."""
    if n <= _CHUNK:
        ctypes.memmove(dst, src, n)
        return
    parts = min((n + _CHUNK - 1) // _CHUNK, 4 * (os.cpu_count() or 1))
    step = (n + parts - 1) // parts
    futs = [_pool().submit(ctypes.memmove, dst + o, src + o, min(step, n - o)) for o in range(0, n, step)]
    for f in futs:
        f.result()


def bytes_address(b: bytes) -> int:
    return _bytes_ptr(b)


def fill_from(dst: torch.Tensor, src: bytes, offset: int = 0) -> None:
    """Copy len(dst) bytes of ``src`` starting at ``offset`` into a CPU uint8 tensor."""
    n = dst.numel()
    if offset + n > len(src):
        raise ValueError("source too short")
    memcpy(dst.data_ptr(), bytes_address(src) + offset, n)


def to_bytes(src: torch.Tensor, header: bytes = b"") -> bytes:
    """A new ``bytes`` = header + the contents of a CPU uint8 tensor (one parallel copy)."""
    n = src.numel()
    out = _new_bytes(None, len(header) + n)  # uninitialised, not yet shared
    base = bytes_address(out)
    if header:
        ctypes.memmove(base, header, len(header))
    memcpy(base + len(header), src.data_ptr(), n)
    return out


def upload(src: bytes, offset: int, nbytes: int, dev: torch.device, slot: str = "in") -> torch.Tensor:
    """``src[offset:offset+nbytes]`` as a new uint8 CUDA tensor (through the pinned buffer)."""
    h = pinned(nbytes, slot)
    fill_from(h, src, offset)
    d = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=dev)[:nbytes]
    d.copy_(h, non_blocking=True)
    return d


def download(parts, header: bytes = b"", slot: str = "out") -> bytes:
    """header + the bytes of the given CUDA tensors, in order, as one ``bytes``.

    Synchronises the current stream (the pinned buffer is reused by the next call)."""
    parts = [p.reshape(-1).view(torch.uint8) for p in parts]
    total = sum(p.numel() for p in parts)
    h = pinned(total, slot)
    o = 0
    for p in parts:
        if p.numel():
            h[o:o + p.numel()].copy_(p, non_blocking=True)
            o += p.numel()
    dev = parts[0].device if parts else device()
    torch.cuda.current_stream(dev).synchronize()
    return to_bytes(h, header)
