"""Codec and Allocator protocols (ashkv/contracts/protocols.py:18-75 of the reference).

Codec: bytes-in/bytes-out ``encode``/``decode`` plus an integer ``checksum``.
Allocator: ``alloc`` returns -1 on failure, ``read`` returns b"" for an
unknown handle, ``pressure`` is a scalar in [0, 1]; none of them raise.
"""
from __future__ import annotations

from typing import Protocol, runtime_checkable

from .tiers import Tier


@runtime_checkable
class Codec(Protocol):
    def encode(self, source_bytes: bytes) -> bytes: ...

    def decode(self, target_bytes: bytes) -> bytes: ...

    def checksum(self, raw_bytes: bytes) -> int: ...


@runtime_checkable
class Allocator(Protocol):
    def alloc(self, tier: Tier, size_bytes: int) -> int: ...

    def free(self, handle: int) -> None: ...

    def read(self, handle: int) -> bytes: ...

    def write(self, handle: int, data: bytes) -> None: ...

    def pressure(self) -> float: ...
