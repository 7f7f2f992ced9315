"""Codecs on sm_100a, registered under the reference's names.

``ashkv/codecs/__init__.py:26-32`` of the reference registers ``bf16``,
``int8_default``, ``int4_default``, ``int2_dithered``, ``nbit_dithered`` and
``fp8_default``; this package registers the same names.
"""
from __future__ import annotations

from ..compiler.registry import codec_registry
from .bf16 import BF16Codec
from .checksum import checksum, checksum_pages, checksum_pair
from .fp8 import FP8Codec
from .int2_dithered import DitheredINT2Codec
from .int4 import INT4Codec
from .int8 import INT8Codec
from .nbit_dithered import DitheredNBitCodec

codec_registry.register("bf16", BF16Codec())
codec_registry.register("int8_default", INT8Codec())
codec_registry.register("int4_default", INT4Codec())
codec_registry.register("int2_dithered", DitheredINT2Codec())
codec_registry.register("nbit_dithered", DitheredNBitCodec())
codec_registry.register("fp8_default", FP8Codec())

__all__ = ["BF16Codec", "FP8Codec", "INT8Codec", "INT4Codec", "DitheredINT2Codec", "DitheredNBitCodec",
           "checksum", "checksum_pair", "checksum_pages"]
