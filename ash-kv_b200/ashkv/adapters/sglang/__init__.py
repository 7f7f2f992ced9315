"""SGLang HiCache adapter: demote/promote hooks, patcher, shadow allocator."""
from __future__ import annotations
