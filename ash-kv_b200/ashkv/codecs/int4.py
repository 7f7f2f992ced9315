"""INT4 group codec on sm_100a.

Drop-in for ``INT4Codec`` (ashkv/codecs/int4.py:19-116 of the reference):
same constructor (``group_size=64``), same blob
``<II num_groups, num_values> + bf16 scale[num_groups] + packed nibbles``
(``num_values`` is the zero-padded count; the even element of each byte in
the high nibble), same empty-input results (``encode(b"")`` is
``<I 0>``; a blob shorter than 8 bytes or with ``num_groups == 0`` decodes
to ``b""``), and decode returns every padded value, as the reference does.
The reference computes in numpy on the host; ``ashkv_int4_encode`` /
``ashkv_int4_decode`` reproduce its bytes, including numpy's int8 cast of
non-finite quotients (0) and torch's CPU bf16 NaN (0xFFFF).

``encode_tensor`` / ``decode_tensor`` are the device-resident entry points.
"""
from __future__ import annotations

import struct
from typing import Optional

import torch

from .. import _native, _staging
from .checksum import checksum


def encode_tensor(src: torch.Tensor, group_size: int = 64, *, scales: Optional[torch.Tensor] = None,
                  packed: Optional[torch.Tensor] = None) -> tuple[torch.Tensor, torch.Tensor, int]:
    """bf16 CUDA tensor (flattened) -> (bf16 scales [n_groups], uint8 packed, num_values)."""
    src = src.contiguous().reshape(-1)
    n_groups = -(-src.numel() // group_size)
    total = n_groups * group_size
    if total % 2:
        raise ValueError(f"operands could not be broadcast together with shapes ({total // 2 + 1},) "
                         f"({total // 2},)")
    if scales is None:
        scales = torch.empty(n_groups, dtype=torch.bfloat16, device=src.device)
    if packed is None:
        packed = torch.empty(total // 2, dtype=torch.uint8, device=src.device)
    _native.int4_encode(src, group_size, scales, packed)
    return scales, packed, total


def decode_tensor(scales: torch.Tensor, packed: torch.Tensor, group_size: int = 64,
                  out: Optional[torch.Tensor] = None) -> torch.Tensor:
    n_groups = scales.numel()
    if out is None:
        out = torch.empty(n_groups * group_size, dtype=torch.bfloat16, device=scales.device)
    _native.int4_decode(scales, packed, n_groups, group_size, out)
    return out


class INT4Codec:
    """INT4 codec with one bf16 absmax scale per ``group_size`` values."""

    __slots__ = ("_encode_calls", "_decode_calls", "_group_size")

    def __init__(self, group_size: int = 64) -> None:
        self._encode_calls = 0
        self._decode_calls = 0
        self._group_size = group_size

    def encode(self, source_bytes: bytes) -> bytes:
        self._encode_calls += 1
        if not source_bytes:
            return struct.pack("<I", 0)
        _staging.check_even(source_bytes)
        gs = self._group_size
        dev = _staging.device()
        src = _staging.upload(source_bytes, 0, len(source_bytes), dev).view(torch.bfloat16)
        scales, packed, total = encode_tensor(src, gs)
        return _staging.download([scales, packed], struct.pack("<II", scales.numel(), total))

    def decode(self, target_bytes: bytes) -> bytes:
        self._decode_calls += 1
        if len(target_bytes) < 8:
            return b""
        num_groups, num_values = struct.unpack("<II", target_bytes[:8])
        if num_groups == 0:
            return b""
        gs = self._group_size
        packed_size = num_values // 2
        avail = max(0, min(packed_size, len(target_bytes) - 8 - 2 * num_groups))
        if len(target_bytes) < 8 + 2 * num_groups:
            raise ValueError(f"INT4 blob too short for {num_groups} scales")
        if 2 * avail != num_groups * gs:
            raise ValueError(f"cannot reshape array of size {2 * avail} into shape ({num_groups},{gs})")
        dev = _staging.device()
        body = _staging.upload(target_bytes, 8, 2 * num_groups + avail, dev)
        out = decode_tensor(body[:2 * num_groups].view(torch.bfloat16), body[2 * num_groups:], gs)
        return _staging.download([out])

    def checksum(self, raw_bytes: bytes) -> int:
        return checksum(raw_bytes)
