"""Hot-path runtime: GPU score/controller, migration ladder, mock allocator."""
from __future__ import annotations

from .allocator import MockAllocator
from .controller import desired_tiers
from .migrate import CodecTable, migrate
from .score import score_vectorized

__all__ = ["score_vectorized", "desired_tiers", "migrate", "CodecTable", "MockAllocator"]
