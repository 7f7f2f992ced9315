"""The eight-number policy configuration (ashkv/contracts/config.py:16-83 of the reference)."""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True, slots=True)
class ASHKVConfig:
    w_T: float = 0.7
    w_S: float = 0.1
    w_N: float = 0.1
    w_P: float = 0.1
    theta_high: float = 0.72
    theta_low: float = 0.33
    delta: float = 0.04
    p_emergency: float = 0.95

    def __post_init__(self) -> None:
        weights = {"w_T": self.w_T, "w_S": self.w_S, "w_N": self.w_N, "w_P": self.w_P}
        total = sum(weights.values())
        if abs(total - 1.0) > 1e-6:
            raise ValueError(
                f"Score weights must sum to 1.0, got {total!r} "
                f"(w_T={self.w_T}, w_S={self.w_S}, w_N={self.w_N}, w_P={self.w_P})")
        for name, v in weights.items():
            if not 0.0 <= v <= 1.0:
                raise ValueError(f"{name} must be in [0, 1], got {v!r}")
        for name in ("theta_high", "theta_low"):
            v = getattr(self, name)
            if not 0.0 <= v <= 1.0:
                raise ValueError(f"{name} must be in [0, 1], got {v!r}")
        if self.theta_low >= self.theta_high:
            raise ValueError(f"theta_low ({self.theta_low!r}) must be strictly less than "
                             f"theta_high ({self.theta_high!r})")
        if self.delta < 0.0:
            raise ValueError(f"delta must be >= 0, got {self.delta!r}")
        if not 0.0 < self.p_emergency < 1.0:
            raise ValueError(f"p_emergency must be in (0, 1), got {self.p_emergency!r}")

    def as_dict(self) -> dict[str, float]:
        return {k: getattr(self, k) for k in ("w_T", "w_S", "w_N", "w_P", "theta_high", "theta_low",
                                              "delta", "p_emergency")}
