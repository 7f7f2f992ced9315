"""score_vectorized on the GPU.

Signature and never-raise contract of ashkv/runtime/score.py:15-52 in the
reference: mismatched or empty inputs return an empty float32 array.  The
arithmetic runs in the ``ashkv_score`` kernel.  numpy inputs are uploaded and
the result downloaded (numpy in, numpy out); CUDA tensors stay on the device.
"""
from __future__ import annotations

import numpy as np
import torch

from .. import _native


def _as_device_f32(a, dev: torch.device) -> torch.Tensor:
    if isinstance(a, torch.Tensor):
        return a.to(device=dev, dtype=torch.float32).contiguous()
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dev)


def score_vectorized(T, S, N, P, w_T: float, w_S: float, w_N: float, w_P: float):
    n = len(T)
    on_gpu = isinstance(T, torch.Tensor) and T.is_cuda
    if not (len(S) == len(N) == len(P) == n) or n == 0:
        return torch.zeros(0, dtype=torch.float32, device=T.device) if on_gpu else np.zeros(0, dtype=np.float32)
    dev = T.device if on_gpu else torch.device("cuda", torch.cuda.current_device())
    Td, Sd, Nd, Pd = (_as_device_f32(a, dev) for a in (T, S, N, P))
    R = torch.empty(n, dtype=torch.float32, device=dev)
    _native.score(Td, Sd, Nd, Pd, float(np.float32(w_T)), float(np.float32(w_S)), float(np.float32(w_N)),
                  float(np.float32(w_P)), R)
    return R if on_gpu else R.cpu().numpy()
