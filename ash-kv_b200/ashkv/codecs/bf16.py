"""BF16 identity codec (ashkv/codecs/bf16.py:16-44 of the reference).

The fallback tier's codec: bytes pass through unchanged; the checksum is
SHA-256 truncated to 8 little-endian bytes, as in the reference.
"""
from __future__ import annotations

from .checksum import _sha8


class BF16Codec:
    __slots__ = ()

    def encode(self, source_bytes: bytes) -> bytes:
        return source_bytes

    def decode(self, target_bytes: bytes) -> bytes:
        return target_bytes

    def checksum(self, raw_bytes: bytes) -> int:
        return _sha8(raw_bytes)
