"""Attention-derived page features: the S (saliency) and N (novelty) inputs of
``score_vectorized`` (ashkv/runtime/score.py:15-52 of the reference), computed
on sm_100a.

The reference produces saliency only inside its simulator
(ashkv/tests/simulator.py:66-80): the causal softmax attention mass that each
key receives, summed over heads and queries.  :func:`attention_saliency`
computes exactly that quantity per token with tensor-core (tcgen05) kernels;
:func:`page_features` turns it into one value per page (the page's mass over
the largest page's mass) and adds the novelty input the reference's config
describes as "key-delta" (``contracts/config.py:26``): the mean over the page
of ||k_t - k_{t-1}||^2 / (||k_t||^2 + ||k_{t-1}||^2) / 2.  Both lie in [0, 1].
"""
from __future__ import annotations

import math
from typing import Optional

import torch

from .. import _native


def attention_saliency(q: torch.Tensor, k: torch.Tensor, *, q_pos0: Optional[int] = None,
                       scale: Optional[float] = None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Attention mass per key: q [n_q, heads_q, head_dim], k [n_k, heads_kv, head_dim] (bf16, CUDA).

    Query i sits at position ``q_pos0 + i`` (default ``n_k - n_q``: the queries
    are the last tokens) and attends keys at positions <= its own.  ``scale``
    defaults to 1/sqrt(head_dim).  Returns fp32 [n_k]."""
    n_q, n_k, d = q.shape[0], k.shape[0], q.shape[2]
    if q_pos0 is None:
        q_pos0 = n_k - n_q
    if scale is None:
        scale = 1.0 / math.sqrt(d)
    if out is None:
        out = torch.empty(n_k, dtype=torch.float32, device=k.device)
    scratch = torch.empty(max(_native.saliency_scratch_floats(q.shape[1], n_q, n_k), 1), dtype=torch.float32,
                          device=k.device)
    status = torch.zeros(1, dtype=torch.int32, device=k.device)
    _native.attention_saliency(q.contiguous(), k.contiguous(), int(q_pos0), float(scale), scratch, out, status)
    return out


def page_features(k: torch.Tensor, tokens_per_page: int = 16, *,
                  token_saliency: Optional[torch.Tensor] = None) -> tuple[Optional[torch.Tensor], torch.Tensor]:
    """(S, N) per page of ``tokens_per_page`` keys; S is None without ``token_saliency``."""
    n_k = k.shape[0]
    n_pages = -(-n_k // tokens_per_page)
    dev = k.device
    N = torch.empty(max(n_pages, 1), dtype=torch.float32, device=dev)
    S = s_raw = None
    if token_saliency is not None:
        S = torch.empty(max(n_pages, 1), dtype=torch.float32, device=dev)
        s_raw = torch.empty(max(n_pages, 1), dtype=torch.float32, device=dev)
    _native.page_features(token_saliency, k.contiguous(), tokens_per_page, s_raw, S, N)
    return (None if S is None else S[:n_pages]), N[:n_pages]


def page_inputs(q: torch.Tensor, k: torch.Tensor, tokens_per_page: int = 16,
                q_pos0: Optional[int] = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Saliency and novelty page inputs of one sequence's layer (queries attend causally)."""
    sal = attention_saliency(q, k, q_pos0=q_pos0)
    S, N = page_features(k, tokens_per_page, token_saliency=sal)
    return S, N
