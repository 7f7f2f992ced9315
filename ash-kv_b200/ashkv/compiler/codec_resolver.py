"""Codec resolver: CodecConfig + hardware + registry -> {(from_tier, to_tier): codec}.

Restates ``resolve_codecs`` (ashkv/compiler/codec_resolver.py:25-156 of the
reference): slot 1 (BF16 <-> FP8 tier) is ``fp8_default`` on hardware with
native FP8, else ``int8_default``; slot 2 (FP8 <-> INT4, plus BF16 <-> INT4
when slot 1 exists) defaults to ``int4_default``; slot 3 (INT4 <-> ARCHIVE)
and slot 4 (ARCHIVE <-> CPU) are off unless named.  "auto" picks the default,
a name picks that registry entry, None disables the slot; a name the registry
does not hold leaves the slot empty (logged).  The reference's slot-3 "auto"
default names ``lowrank_default``, which its registry never registers, so
"auto" there also leaves the slot empty.

``page_format(codec)`` maps a codec to the page format the batched migration
(``ashkv.runtime.batch``) stores for its tier.
"""
from __future__ import annotations

import logging
from dataclasses import dataclass
from typing import Optional

from ..contracts.protocols import Codec
from ..contracts.tiers import Tier
from .hardware_probe import HardwareProfile
from .registry import CodecRegistry, codec_registry

logger = logging.getLogger("ashkv.compiler.codec_resolver")


@dataclass(frozen=True, slots=True)
class CodecConfig:
    bf16_to_compressed: Optional[str] = "auto"
    compressed_to_cold: Optional[str] = "auto"
    cold_to_archive: Optional[str] = None
    archive_to_cpu: Optional[str] = None


def _slot(user: Optional[str], default: Optional[str]) -> Optional[str]:
    if user is None:
        return None
    return default if user == "auto" else user


def _get(name: str, registry: CodecRegistry, slot: str) -> Optional[Codec]:
    codec = registry.get(name)
    if codec is None:
        logger.warning("codec '%s' requested for slot '%s' is not registered; the slot is unavailable", name, slot)
    return codec


def resolve_codecs(codec_config: CodecConfig, hardware: HardwareProfile,
                   registry: CodecRegistry = codec_registry) -> dict[tuple[int, int], Codec]:
    table: dict[tuple[int, int], Codec] = {}
    bf16, fp8, int4, archive, cpu = (int(t) for t in (Tier.BF16, Tier.FP8, Tier.INT4, Tier.ARCHIVE, Tier.CPU))
    default1 = "fp8_default" if hardware.has_fp8_native else "int8_default"
    if not hardware.has_fp8_native and not hardware.has_int8_native:
        logger.warning("no FP8 or INT8 hardware acceleration detected; using INT8")
    name = _slot(codec_config.bf16_to_compressed, default1)
    if name is not None and (c := _get(name, registry, "bf16_to_compressed")) is not None:
        table[(bf16, fp8)] = table[(fp8, bf16)] = c
    name = _slot(codec_config.compressed_to_cold, "int4_default")
    if name is not None and (c := _get(name, registry, "compressed_to_cold")) is not None:
        table[(fp8, int4)] = table[(int4, fp8)] = c
        if (bf16, fp8) in table:
            table[(bf16, int4)] = table[(int4, bf16)] = c
    name = _slot(codec_config.cold_to_archive, "lowrank_default")
    if name is not None and (c := _get(name, registry, "cold_to_archive")) is not None:
        table[(int4, archive)] = table[(archive, int4)] = c
    name = _slot(codec_config.archive_to_cpu, None)
    if name is not None and (c := _get(name, registry, "archive_to_cpu")) is not None:
        table[(archive, cpu)] = table[(cpu, archive)] = c
    for (a, b), c in sorted(table.items()):
        logger.info("  %s -> %s: %s", Tier(a).name, Tier(b).name, type(c).__name__)
    return table


def page_format(codec) -> int:
    """Page format of the batched migration for a codec instance (-1 if it has none)."""
    from .. import _native
    from ..codecs import bf16 as _bf16, fp8 as _fp8, int4 as _int4, int8 as _int8, nbit_dithered as _nb
    if isinstance(codec, _int8.INT8Codec):
        return _native.PAGE_INT8
    if isinstance(codec, _fp8.FP8Codec):
        return _native.PAGE_FP8
    if isinstance(codec, _int4.INT4Codec):
        return _native.PAGE_INT4 if getattr(codec, "_group_size", 64) == 64 else _native.PAGE_NONE
    if isinstance(codec, _nb.DitheredNBitCodec):
        bits = getattr(codec, "_bits", 4)
        return {4: _native.PAGE_NBIT4, 2: _native.PAGE_NBIT2}.get(bits, _native.PAGE_NONE)
    if isinstance(codec, _bf16.BF16Codec):
        return _native.PAGE_BF16
    return _native.PAGE_NONE


def tier_formats(table: dict[tuple[int, int], Codec]) -> dict[int, int]:
    """Tier -> page format: each tier stores pages with the codec of the edge that enters it from the
    next hotter tier (BF16 pages stay in the KV pool)."""
    out = {int(Tier.BF16): 0}
    for t in (Tier.FP8, Tier.INT4, Tier.ARCHIVE):
        t = int(t)
        codec = table.get((t - 1, t))
        if codec is not None:
            out[t] = page_format(codec)
    return out
