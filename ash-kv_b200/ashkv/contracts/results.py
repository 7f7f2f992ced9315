"""Typed, never-raised results of hot-path operations.

Same enums and dataclasses as ashkv/contracts/results.py:21-64 of the
reference (the integer values are consumed by telemetry and tests).
"""
from __future__ import annotations

from dataclasses import dataclass
from enum import IntEnum

from .tiers import Tier


class MigrationStatus(IntEnum):
    OK = 0
    SKIPPED = 1
    FAILURE = 2
    FALLBACK = 3
    CORRUPT = 4


class PressureState(IntEnum):
    NORMAL = 0
    ELEVATED = 1
    CRITICAL = 2
    SATURATED = 3


PRESSURE_ELEVATED_THRESHOLD: float = 0.85
PRESSURE_SATURATED_THRESHOLD: float = 0.99


@dataclass(slots=True, frozen=True)
class MigrationResult:
    status: MigrationStatus
    page_id: int
    from_tier: Tier
    to_tier: Tier
    duration_us: int
    error: str = ""


@dataclass(slots=True, frozen=True)
class PressureReport:
    pressure: float
    state: PressureState
