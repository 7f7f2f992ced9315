"""FP8 (E4M3FN) codec on sm_100a.

Drop-in for ``FP8Codec`` (ashkv/codecs/fp8.py:17-83 of the reference): no
header, one float8_e4m3fn byte per bf16 input element; empty input encodes
and decodes to ``b""``; the checksum is the shared ``checksum``.  The
reference casts with torch (``tensor.to(torch.float8_e4m3fn)`` and back, on
the GPU when one is present); ``ashkv_fp8_encode`` / ``ashkv_fp8_decode``
compute the same bytes: round to nearest even with no saturation (|x| > 464,
inf and NaN become NaN), NaN decoded as bf16 0x7FFF.

``encode_tensor`` / ``decode_tensor`` are the device-resident entry points.
"""
from __future__ import annotations

from typing import Optional

import torch

from .. import _native, _staging
from .checksum import checksum


def encode_tensor(src: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """bf16 CUDA tensor -> uint8 tensor of float8_e4m3fn codes (same shape)."""
    src = src.contiguous()
    if out is None:
        out = torch.empty(src.shape, dtype=torch.uint8, device=src.device)
    _native.fp8_encode(src, out)
    return out


def decode_tensor(codes: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """uint8 / float8_e4m3fn CUDA tensor -> bf16 tensor (same shape)."""
    codes = codes.contiguous()
    if out is None:
        out = torch.empty(codes.shape, dtype=torch.bfloat16, device=codes.device)
    _native.fp8_decode(codes, out)
    return out


class FP8Codec:
    """FP8 (E4M3FN) codec: bf16 bytes <-> one code byte per element."""

    __slots__ = ("_encode_calls", "_decode_calls")

    def __init__(self) -> None:
        self._encode_calls = 0
        self._decode_calls = 0

    def encode(self, source_bytes: bytes) -> bytes:
        self._encode_calls += 1
        if not source_bytes:
            return b""
        _staging.check_even(source_bytes)
        dev = _staging.device()
        src = _staging.upload(source_bytes, 0, len(source_bytes), dev).view(torch.bfloat16)
        return _staging.download([encode_tensor(src)])

    def decode(self, target_bytes: bytes) -> bytes:
        self._decode_calls += 1
        if not target_bytes:
            return b""
        dev = _staging.device()
        codes = _staging.upload(target_bytes, 0, len(target_bytes), dev)
        return _staging.download([decode_tensor(codes)])

    def checksum(self, raw_bytes: bytes) -> int:
        return checksum(raw_bytes)
