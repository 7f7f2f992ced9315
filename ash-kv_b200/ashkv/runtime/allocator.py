"""In-memory allocator for tests and host-only integration (Allocator protocol).

Mirrors ``MockAllocator`` (ashkv/runtime/allocator.py:18-125 of the
reference): a dict of byte buffers with a byte budget; ``alloc`` of a
non-positive size or past the budget returns -1; ``pressure`` is used/budget
clamped to [0, 1].
"""
from __future__ import annotations

from ..contracts.tiers import Tier


class MockAllocator:
    __slots__ = ("_buffers", "_next_handle", "_budget", "_used", "_per_tier_used", "_handle_to_tier")

    def __init__(self, budget_bytes: int = 10 * 1024 * 1024 * 1024) -> None:
        self._buffers: dict[int, bytes] = {}
        self._next_handle = 1
        self._budget = budget_bytes
        self._used = 0
        self._per_tier_used: dict[int, int] = {}
        self._handle_to_tier: dict[int, int] = {}

    def alloc(self, tier: Tier, size_bytes: int) -> int:
        if size_bytes <= 0 or self._used + size_bytes > self._budget:
            return -1
        h = self._next_handle
        self._next_handle += 1
        self._buffers[h] = b"\x00" * size_bytes
        self._used += size_bytes
        self._per_tier_used[int(tier)] = self._per_tier_used.get(int(tier), 0) + size_bytes
        self._handle_to_tier[h] = int(tier)
        return h

    def free(self, handle: int) -> None:
        buf = self._buffers.pop(handle, None)
        if buf is None:
            return
        self._used -= len(buf)
        t = self._handle_to_tier.pop(handle, None)
        if t is not None:
            self._per_tier_used[t] = self._per_tier_used.get(t, 0) - len(buf)

    def read(self, handle: int) -> bytes:
        return self._buffers.get(handle, b"")

    def write(self, handle: int, data: bytes) -> None:
        if handle not in self._buffers:
            return
        old = len(self._buffers[handle])
        self._buffers[handle] = bytes(data)
        delta = len(data) - old
        self._used += delta
        t = self._handle_to_tier.get(handle)
        if t is not None:
            self._per_tier_used[t] = self._per_tier_used.get(t, 0) + delta

    def pressure(self) -> float:
        if self._budget <= 0:
            return 1.0
        return max(0.0, min(1.0, self._used / self._budget))

    @property
    def used_bytes(self) -> int:
        return self._used

    @property
    def budget_bytes(self) -> int:
        return self._budget

    def tier_usage(self, tier: Tier) -> int:
        return self._per_tier_used.get(int(tier), 0)

    @property
    def num_allocations(self) -> int:
        return len(self._buffers)

    # -- test utilities (outside the Allocator protocol) -----------------------
    def reset(self) -> None:
        self._buffers.clear()
        self._handle_to_tier.clear()
        self._per_tier_used.clear()
        self._next_handle = 1
        self._used = 0

    def set_budget(self, budget: int) -> None:
        self._budget = budget

    def preload(self, handle: int, data: bytes, tier: Tier = Tier.BF16) -> None:
        """Place ``data`` at a chosen handle (test setup)."""
        self._buffers[handle] = data
        self._used += len(data)
        self._per_tier_used[int(tier)] = self._per_tier_used.get(int(tier), 0) + len(data)
        self._handle_to_tier[handle] = int(tier)
        self._next_handle = max(self._next_handle, handle + 1)
