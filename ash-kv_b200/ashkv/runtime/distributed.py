"""The one cross-rank exchange of the tiering policy: allocator pressure.

Pages are sharded across ranks along KV heads while the page table is
replicated, so every rank must evaluate ``desired_tiers`` with the same
pressure scalar or the ranks would demote different pages.  Each rank
contributes its local allocator pressure and all use the maximum (the most
constrained rank decides).  A 4-byte all-reduce: latency only.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist


def allreduce_pressure(pressure: float, group: Optional[dist.ProcessGroup] = None,
                       device: Optional[torch.device] = None) -> float:
    """MAX of ``pressure`` over the ranks of ``group`` (identity without a process group)."""
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size(group) == 1:
        return float(pressure)
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend(group) == "nccl" \
            else torch.device("cpu")
    t = torch.tensor([float(pressure)], dtype=torch.float32, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
