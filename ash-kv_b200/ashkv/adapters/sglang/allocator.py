"""Shadow-cache allocator backed by one device arena.

Drop-in for ``SGLangShadowAllocator`` (ashkv/adapters/sglang/allocator.py:4-82
of the reference): ``alloc(tier, size) -> handle`` (-1 past the byte budget),
``free``, ``get_tensor`` (a writable uint8 CUDA view of the buffer),
``get_utilization``/``pressure`` (allocated / max), ``read``/``write`` through
host bytes.

Instead of one ``torch.empty`` per handle, every buffer is a 256-byte-aligned
sub-range of a single device arena (allocated on first use), so kernels can
address any handle as ``arena_base + offset``: ``offsets(handles)`` returns
the byte offsets as a device tensor for batched encode/decode kernels.
Freed ranges are recycled by exact size first (pages of one codec share a
size), then best fit; the arena never grows past ``max_bytes``.
"""
from __future__ import annotations

import bisect
from typing import Optional

import numpy as np
import torch

ALIGN = 256


def _round(n: int) -> int:
    return (n + ALIGN - 1) // ALIGN * ALIGN


class SGLangShadowAllocator:
    def __init__(self, max_bytes: int, device: Optional[torch.device] = None):
        self.max_bytes = max_bytes
        self.allocated_bytes = 0
        self.pool: dict[int, tuple[int, int]] = {}  # handle -> (offset, size)
        self.next_handle = 1
        self._device = device
        self._arena: Optional[torch.Tensor] = None
        self._bump = 0
        self._free_by_size: dict[int, list[int]] = {}   # rounded size -> offsets
        self._free_sizes: list[int] = []                 # sorted rounded sizes with free ranges

    # ------------------------------------------------------------------ arena
    @property
    def arena(self) -> torch.Tensor:
        if self._arena is None:
            dev = self._device or torch.device("cuda", torch.cuda.current_device())
            self._arena = torch.empty(_round(max(self.max_bytes, ALIGN)), dtype=torch.uint8, device=dev)
        return self._arena

    def _take(self, rsize: int) -> int:
        lst = self._free_by_size.get(rsize)
        if lst:
            off = lst.pop()
            if not lst:
                self._drop_size(rsize)
            return off
        if self._bump + rsize <= _round(max(self.max_bytes, ALIGN)):
            off = self._bump
            self._bump += rsize
            return off
        i = bisect.bisect_left(self._free_sizes, rsize)
        if i < len(self._free_sizes):  # best fit: split a larger free range
            big = self._free_sizes[i]
            off = self._free_by_size[big].pop()
            if not self._free_by_size[big]:
                self._drop_size(big)
            self._give(off + rsize, big - rsize)
            return off
        return -1

    def _give(self, off: int, rsize: int) -> None:
        if rsize <= 0:
            return
        lst = self._free_by_size.get(rsize)
        if lst is None:
            self._free_by_size[rsize] = [off]
            bisect.insort(self._free_sizes, rsize)
        else:
            lst.append(off)

    def _drop_size(self, rsize: int) -> None:
        del self._free_by_size[rsize]
        i = bisect.bisect_left(self._free_sizes, rsize)
        del self._free_sizes[i]

    # ------------------------------------------------------------------ protocol
    def alloc(self, tier, size_bytes: int) -> int:
        if size_bytes <= 0 or self.allocated_bytes + size_bytes > self.max_bytes:
            return -1
        off = self._take(_round(size_bytes))
        if off < 0:
            return -1
        h = self.next_handle
        self.next_handle += 1
        self.pool[h] = (off, size_bytes)
        self.allocated_bytes += size_bytes
        return h

    def alloc_many(self, tier, size_bytes: int, count: int) -> np.ndarray:
        """``count`` handles of one size (-1 where the budget runs out)."""
        return np.array([self.alloc(tier, size_bytes) for _ in range(count)], dtype=np.int64)

    def free(self, handle: int) -> None:
        ent = self.pool.pop(handle, None)
        if ent is None:
            return
        off, size = ent
        self.allocated_bytes -= size
        self._give(off, _round(size))

    def get_tensor(self, handle: int) -> torch.Tensor | None:
        ent = self.pool.get(handle)
        if ent is None:
            return None
        off, size = ent
        return self.arena[off:off + size]

    def offsets(self, handles) -> torch.Tensor:
        """Byte offsets of ``handles`` within the arena, as an int64 device tensor."""
        offs = np.array([self.pool[int(h)][0] for h in handles], dtype=np.int64)
        return torch.from_numpy(offs).to(self.arena.device)

    def get_utilization(self) -> float:
        if self.max_bytes == 0:
            return 0.0
        return self.allocated_bytes / self.max_bytes

    def read(self, handle: int) -> bytes:
        t = self.get_tensor(handle)
        if t is None:
            return b""
        return t.cpu().numpy().tobytes()

    def write(self, handle: int, data: bytes) -> None:
        t = self.get_tensor(handle)
        if t is None:
            return
        src = torch.from_numpy(np.frombuffer(data, dtype=np.uint8).copy())
        t[: len(data)].copy_(src)

    def pressure(self) -> float:
        return self.get_utilization()
