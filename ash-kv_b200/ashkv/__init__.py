"""ashkv — B200-native KV-page codec and demote/promote path for ASH-KV.

Drop-in for the reference package's hot-path API: the ``ashkv.codecs``
registry, ``ashkv.runtime`` (``score_vectorized``, ``desired_tiers``,
``migrate``), the SGLang ``demote_hook``/``promote_hook`` and
``SGLangShadowAllocator``.  The arithmetic runs in sm_100a CUDA kernels in
``ashkv/_lib/libashkv_cuda.so`` (built from ``csrc/``), loaded through
``ashkv._native``; there is no CPU fallback for the codec kernels.
"""
from __future__ import annotations

__version__ = "0.1.0"
