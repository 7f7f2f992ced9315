"""ASH-KV contracts: tiers, page table, policy config, protocols, typed results."""
from __future__ import annotations

from .config import ASHKVConfig
from .page import PAGE_DTYPE, PageHandle, PageTable
from .protocols import Allocator, Codec
from .results import (
    PRESSURE_ELEVATED_THRESHOLD,
    PRESSURE_SATURATED_THRESHOLD,
    MigrationResult,
    MigrationStatus,
    PressureReport,
    PressureState,
)
from .tiers import (
    COLDEST_TIER,
    HOTTEST_TIER,
    NUM_TIERS,
    Tier,
    is_colder,
    is_hotter,
    next_colder,
    next_hotter,
    tier_distance,
)

__all__ = [
    "Tier", "NUM_TIERS", "HOTTEST_TIER", "COLDEST_TIER", "is_hotter", "is_colder", "next_hotter",
    "next_colder", "tier_distance", "PageTable", "PageHandle", "PAGE_DTYPE", "ASHKVConfig",
    "MigrationStatus", "PressureState", "MigrationResult", "PressureReport",
    "PRESSURE_ELEVATED_THRESHOLD", "PRESSURE_SATURATED_THRESHOLD", "Codec", "Allocator",
]
