"""Single-page migration ladder.

Same contract, ladder and status/error strings as ``migrate`` in
ashkv/runtime/migrate.py:35-191 of the reference (the strings are asserted by
callers' tests): pin -> no-op -> codec lookup -> breaker -> read -> encode ->
alloc -> write -> verify (checksum of decode(encoded) against the page's
bf16 checksum) -> commit -> free source.  Never raises.

As in the reference, the same codec serves both directions of a tier pair and
``encode`` is applied for promotions too.  For many pages at once use
``ashkv.runtime.batch.migrate_pages``, which runs the gather/encode/verify
steps as fused kernels.
"""
from __future__ import annotations

import time
from typing import Any, Callable

from ..contracts.page import PageTable
from ..contracts.protocols import Allocator, Codec
from ..contracts.results import MigrationResult, MigrationStatus
from ..contracts.tiers import Tier

CodecTable = dict[tuple[int, int], Codec]


def _call(fn: Callable, *args, default=None):
    try:
        return fn(*args)
    except Exception:
        return default


def migrate(page_id: int, target_tier: Tier, page_table: PageTable, allocator: Allocator,
            codec_table: CodecTable, page_handle_lookup: Callable[[int], int],
            page_size_lookup: Callable[[int], int], breaker_registry: Any = None) -> MigrationResult:
    t0 = time.perf_counter_ns()

    def done(status: MigrationStatus, frm: Tier, to: Tier, err: str = "") -> MigrationResult:
        return MigrationResult(status=status, page_id=page_id, from_tier=frm, to_tier=to,
                               duration_us=int((time.perf_counter_ns() - t0) // 1000), error=err)

    raw = page_table.get_tier(page_id)
    if raw < 0:
        return done(MigrationStatus.SKIPPED, Tier.BF16, target_tier, "page not found")
    cur = Tier(raw)
    pins = page_table.get_pin_count(page_id)
    if pins < 0:
        return done(MigrationStatus.SKIPPED, cur, target_tier, "page not found")
    if pins > 0:
        return done(MigrationStatus.SKIPPED, cur, target_tier, "pinned")
    if cur == target_tier:
        return done(MigrationStatus.SKIPPED, cur, target_tier, "already at target")
    codec = codec_table.get((int(cur), int(target_tier)))
    if codec is None:
        return done(MigrationStatus.SKIPPED, cur, target_tier, "no codec")
    name = f"{cur.name}_to_{target_tier.name}"
    if breaker_registry is not None and not breaker_registry.is_codec_available(name):
        return done(MigrationStatus.SKIPPED, cur, target_tier, "breaker tripped")

    def fail_codec() -> None:
        if breaker_registry is not None:
            breaker_registry.record_codec_failure(name)

    src_handle = _call(page_handle_lookup, page_id, default=-1)
    if src_handle < 0:
        return done(MigrationStatus.FAILURE, cur, target_tier, "no handle")
    src = _call(allocator.read, src_handle, default=None)
    if src is None:
        return done(MigrationStatus.FAILURE, cur, target_tier, "read failed")
    try:
        enc = codec.encode(src)
    except Exception as e:
        fail_codec()
        return done(MigrationStatus.FAILURE, cur, target_tier, f"encode: {e}")
    dst_handle = _call(allocator.alloc, target_tier, len(enc), default=-1)
    if dst_handle < 0:
        return done(MigrationStatus.FAILURE, cur, target_tier, "alloc failed")
    try:
        allocator.write(dst_handle, enc)
    except Exception:
        _call(allocator.free, dst_handle)
        return done(MigrationStatus.FAILURE, cur, target_tier, "write failed")
    try:
        back = codec.decode(enc)
    except Exception as e:
        _call(allocator.free, dst_handle)
        fail_codec()
        return done(MigrationStatus.FAILURE, cur, target_tier, f"verify decode: {e}")
    try:
        digest = codec.checksum(back)
    except Exception as e:
        _call(allocator.free, dst_handle)
        fail_codec()
        return done(MigrationStatus.FAILURE, cur, target_tier, f"verify checksum: {e}")
    if digest != page_table.get_bf16_checksum(page_id):
        _call(allocator.free, dst_handle)
        fail_codec()
        return done(MigrationStatus.CORRUPT, cur, target_tier, "checksum mismatch")
    if not page_table.apply_tier_transition(page_id, target_tier, digest):
        _call(allocator.free, dst_handle)
        return done(MigrationStatus.SKIPPED, cur, target_tier, "commit rejected (pin race)")
    _call(allocator.free, src_handle)
    if breaker_registry is not None:
        breaker_registry.record_codec_success(name)
    return done(MigrationStatus.OK, cur, target_tier)
