"""Safety primitives used on the migration path (circuit breakers)."""
from __future__ import annotations

from .circuit_breaker import CircuitBreaker, CircuitBreakerRegistry

__all__ = ["CircuitBreaker", "CircuitBreakerRegistry"]
