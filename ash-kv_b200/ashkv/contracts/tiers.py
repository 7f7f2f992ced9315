"""KV residency tiers, ordered hottest (0) to coldest.

Mirrors ``Tier`` and its helpers in ashkv/contracts/tiers.py:18-66 of the
reference: the integer values are part of the wire/page-table format, so they
are identical (BF16=0 ... DISK=5).
"""
from __future__ import annotations

from enum import IntEnum


class Tier(IntEnum):
    BF16 = 0      # exact hot state
    FP8 = 1       # first compression slot (FP8, or INT8 where FP8 is not chosen)
    INT4 = 2      # cold GPU tier
    ARCHIVE = 3   # coldest GPU tier (INT2 dithered)
    CPU = 4       # host offload
    DISK = 5      # persistent storage


NUM_TIERS: int = len(Tier)
HOTTEST_TIER: Tier = Tier.BF16
COLDEST_TIER: Tier = Tier.DISK


def is_hotter(a: Tier, b: Tier) -> bool:
    return int(a) < int(b)


def is_colder(a: Tier, b: Tier) -> bool:
    return int(a) > int(b)


def next_hotter(t: Tier) -> Tier | None:
    return None if t == HOTTEST_TIER else Tier(int(t) - 1)


def next_colder(t: Tier) -> Tier | None:
    return None if t == COLDEST_TIER else Tier(int(t) + 1)


def tier_distance(a: Tier, b: Tier) -> int:
    return abs(int(a) - int(b))
