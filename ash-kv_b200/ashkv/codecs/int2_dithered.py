"""Dithered INT2 codec (ashkv/codecs/int2_dithered.py:13-147 of the reference).

The same arithmetic as the N-bit codec with bits = 2, group 32 and sigma 3,
but the reference seeds its dither generator with a fixed 42 on every call;
this codec keeps that policy for its in-kernel Philox dither.  ``uniform=``
injects the reference's U tensor for bit-exact reproduction.
"""
from __future__ import annotations

from .nbit_dithered import DitheredNBitCodec


class DitheredINT2Codec(DitheredNBitCodec):
    __slots__ = ()

    def __init__(self, hidden_dim: int = 128) -> None:
        super().__init__(hidden_dim=hidden_dim, group_size=32, sigma=3.0, bits=2)

    def _seed(self) -> int:
        return 42
