"""Per-codec circuit breakers.

Behaviour of ashkv/safety/circuit_breaker.py:30-143 in the reference: a
breaker trips when ``threshold`` failures fall inside ``window_seconds``,
stays tripped for ``cooldown_seconds`` (successes do not reset it) and then
resets itself.  Unknown codec names count as available.  Not thread-safe.
"""
from __future__ import annotations

import time
from dataclasses import dataclass, field


@dataclass(slots=True)
class CircuitBreaker:
    threshold: int = 5
    window_seconds: float = 60.0
    cooldown_seconds: float = 60.0
    _failures: list[float] = field(default_factory=list, repr=False)
    _tripped: bool = False
    _tripped_at: float = 0.0

    def _prune(self, now: float) -> None:
        cutoff = now - self.window_seconds
        self._failures = [t for t in self._failures if t >= cutoff]

    @property
    def is_tripped(self) -> bool:
        if not self._tripped:
            return False
        if time.monotonic() - self._tripped_at >= self.cooldown_seconds:
            self._tripped = False
            self._failures.clear()
            return False
        return True

    def record_failure(self) -> None:
        now = time.monotonic()
        self._prune(now)
        self._failures.append(now)
        if not self._tripped and len(self._failures) >= self.threshold:
            self._tripped, self._tripped_at = True, now

    def record_success(self) -> None:
        self._prune(time.monotonic())

    def reset(self) -> None:
        self._tripped = False
        self._failures.clear()
        self._tripped_at = 0.0

    @property
    def failure_count(self) -> int:
        cutoff = time.monotonic() - self.window_seconds
        return sum(1 for t in self._failures if t >= cutoff)


@dataclass(slots=True)
class CircuitBreakerRegistry:
    _breakers: dict[str, CircuitBreaker] = field(default_factory=dict, repr=False)

    def get_or_create(self, codec_name: str) -> CircuitBreaker:
        b = self._breakers.get(codec_name)
        if b is None:
            b = self._breakers[codec_name] = CircuitBreaker()
        return b

    def is_codec_available(self, codec_name: str) -> bool:
        b = self._breakers.get(codec_name)
        return True if b is None else not b.is_tripped

    def record_codec_failure(self, codec_name: str) -> None:
        self.get_or_create(codec_name).record_failure()

    def record_codec_success(self, codec_name: str) -> None:
        b = self._breakers.get(codec_name)
        if b is not None:
            b.record_success()

    def all_breakers(self) -> dict[str, CircuitBreaker]:
        return dict(self._breakers)

    def reset_all(self) -> None:
        for b in self._breakers.values():
            b.reset()
