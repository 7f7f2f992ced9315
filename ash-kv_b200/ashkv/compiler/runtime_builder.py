"""Compile the eight-number config into hot-path closures.

Mirrors ashkv/compiler/runtime_builder.py:41-173 of the reference:
``compile_score`` and ``compile_controller`` capture the config values (the
hot path never reads the config), ``compile_controller`` derives the
next-colder / next-hotter tier lookup tables from the codec table's
``(from, to)`` keys, and ``build_runtime`` assembles a ``CompiledRuntime``.
The closures call the GPU ``score_vectorized`` / ``desired_tiers``.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Iterable

import numpy as np

from ..contracts.config import ASHKVConfig
from ..contracts.results import MigrationResult
from ..contracts.tiers import NUM_TIERS, Tier
from ..runtime.controller import desired_tiers
from ..runtime.migrate import CodecTable, migrate
from ..runtime.score import score_vectorized

ScoreFn = Callable
ControllerFn = Callable
MigrateFn = Callable
TelemetryFn = Callable[[MigrationResult], None]


@dataclass(slots=True, frozen=True)
class CompiledRuntime:
    config: ASHKVConfig
    score_fn: ScoreFn
    controller_fn: ControllerFn
    migrate_fn: MigrateFn
    codec_table: CodecTable
    telemetry_fn: TelemetryFn


def controller_tables(codec_keys: Iterable[tuple[int, int]]) -> tuple[np.ndarray, np.ndarray]:
    """Lookup tables: one tier colder / hotter per tier, restricted to codec-reachable targets."""
    keys = [(int(a), int(b)) for a, b in codec_keys]
    nc = np.array([min(i + 1, NUM_TIERS - 1) for i in range(NUM_TIERS)], dtype=np.int8)
    nh = np.array([max(i - 1, 0) for i in range(NUM_TIERS)], dtype=np.int8)
    for src in range(NUM_TIERS):
        colder = [t for s, t in keys if s == src and t > src]
        hotter = [t for s, t in keys if s == src and t < src]
        if colder:
            nc[src] = min(colder)
        if hotter:
            nh[src] = max(hotter)
    return nc, nh


def compile_score(config: ASHKVConfig) -> ScoreFn:
    w = (config.w_T, config.w_S, config.w_N, config.w_P)

    def score_fn(T, S, N, P):
        return score_vectorized(T, S, N, P, *w)

    return score_fn


def compile_controller(config: ASHKVConfig, codec_table: CodecTable) -> ControllerFn:
    theta_high, theta_low, delta, p_emergency = (config.theta_high, config.theta_low, config.delta,
                                                 config.p_emergency)
    next_colder, next_hotter = controller_tables(codec_table.keys())

    def controller_fn(R, current_tiers, pressure: float):
        return desired_tiers(R, current_tiers, pressure, theta_high, theta_low, delta, p_emergency, next_colder,
                             next_hotter)

    return controller_fn


def compile_migrate() -> MigrateFn:
    return migrate


def compile_telemetry(enabled: bool) -> TelemetryFn:
    if not enabled:
        return lambda _result: None
    counts: dict[int, int] = {}

    def record(result: MigrationResult) -> None:
        counts[int(result.status)] = counts.get(int(result.status), 0) + 1

    record.counts = counts  # type: ignore[attr-defined]
    return record


def build_runtime(config: ASHKVConfig, codec_table: CodecTable, telemetry_enabled: bool = False) -> CompiledRuntime:
    return CompiledRuntime(config=config, score_fn=compile_score(config),
                           controller_fn=compile_controller(config, codec_table), migrate_fn=compile_migrate(),
                           codec_table=codec_table, telemetry_fn=compile_telemetry(telemetry_enabled))


__all__ = ["CompiledRuntime", "build_runtime", "compile_score", "compile_controller", "compile_migrate",
           "compile_telemetry", "controller_tables", "Tier"]
