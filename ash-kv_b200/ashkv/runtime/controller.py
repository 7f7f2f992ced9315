"""desired_tiers on the GPU.

Signature and contract of ashkv/runtime/controller.py:32-106 in the
reference: empty or mismatched inputs return a copy of ``current_tiers``; the
result has the dtype of ``current_tiers``.  The threshold arithmetic (pressure
boost, hysteresis) is done in double precision and the per-page comparison in
the ``ashkv_desired_tiers`` kernel.  numpy in -> numpy out; CUDA tensors stay
on the device.
"""
from __future__ import annotations

import numpy as np
import torch

from .. import _native


def desired_tiers(R, current_tiers, pressure: float, theta_high: float, theta_low: float, delta: float,
                  p_emergency: float, next_colder, next_hotter):
    n = len(R)
    if n == 0 or len(current_tiers) != n:
        if hasattr(current_tiers, "clone") and isinstance(current_tiers, torch.Tensor):
            return current_tiers.clone()
        return current_tiers.copy() if hasattr(current_tiers, "copy") else np.array([], dtype=np.int8)
    on_gpu = isinstance(R, torch.Tensor) and R.is_cuda
    dev = R.device if on_gpu else torch.device("cuda", torch.cuda.current_device())
    if isinstance(R, torch.Tensor):
        Rd = R.to(device=dev, dtype=torch.float32).contiguous()
    else:
        Rd = torch.from_numpy(np.ascontiguousarray(R, dtype=np.float32)).to(dev)
    if isinstance(current_tiers, torch.Tensor):
        out_dtype = current_tiers.dtype
        cur = current_tiers.to(device=dev, dtype=torch.int8).contiguous()
    else:
        out_dtype = np.asarray(current_tiers).dtype
        cur = torch.from_numpy(np.ascontiguousarray(current_tiers, dtype=np.int8)).to(dev)
    target = torch.empty(n, dtype=torch.int8, device=dev)
    _native.desired_tiers(Rd, cur, float(pressure), float(theta_high), float(theta_low), float(delta),
                          float(p_emergency), np.asarray(next_colder), np.asarray(next_hotter), target)
    if on_gpu:
        return target if out_dtype == torch.int8 else target.to(out_dtype)
    return target.cpu().numpy().astype(out_dtype, copy=False)
