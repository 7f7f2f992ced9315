"""GPU tests: attention-derived page features (saliency on tcgen05, novelty).

Saliency is floating-point work: the kernels compute the scores on the
tensor cores with fp32 accumulation and the softmax with exp2, so they are
compared with the oracle's fp32 restatement of the reference simulator
(ashkv/tests/simulator.py:66-80) within a relative tolerance of 1e-4 of the
largest value (observed errors are ~1e-6).  Page features are compared with
the oracle's float64 definitions within 1e-4.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle

from ashkv.runtime import features as F

pytestmark = pytest.mark.gpu

TOL = 1e-4


def qk(n_q, n_k, hq, hkv, d, seed, scale=0.5):
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(n_q, hq, d, generator=g) * scale).to(torch.bfloat16)
    k = (torch.randn(n_k, hkv, d, generator=g) * scale).to(torch.bfloat16)
    return q, k


def close(got: torch.Tensor, want, tol=TOL):
    got = got.detach().cpu().double().numpy()
    want = np.asarray(want, dtype=np.float64)
    assert got.shape == want.shape
    err = np.abs(got - want).max() if got.size else 0.0
    assert err <= tol * max(np.abs(want).max(), 1e-30), err


@pytest.mark.parametrize("n_q,n_k,hq,hkv,d,q_pos0", [
    (1024, 1024, 8, 8, 64, None),       # the simulator's shape (seq 1024, 8 heads x 64)
    (1000, 1000, 32, 8, 128, None),     # GQA, ragged last tile
    (128, 128, 1, 1, 64, None),         # one tile
    (64, 1000, 8, 8, 128, None),        # decode-style: the last 64 queries
    (1, 777, 4, 2, 64, None),           # one query
    (300, 300, 2, 2, 128, -50),         # queries before the keys start (early rows see nothing)
    (512, 256, 2, 2, 64, 0),            # more queries than keys
])
def test_attention_saliency_vs_oracle(cuda, n_q, n_k, hq, hkv, d, q_pos0):
    q, k = qk(n_q, n_k, hq, hkv, d, n_q + n_k + hq + d)
    got = F.attention_saliency(q.to(cuda), k.to(cuda), q_pos0=q_pos0)
    want = oracle.attention_saliency(q, k, q_pos0=q_pos0)
    close(got, want)


def test_saliency_total_mass_and_large_scores(cuda):
    """Each visible query row sums to 1; large logits (scale 4) stay finite."""
    q, k = qk(700, 700, 4, 4, 128, 3, scale=4.0)
    got = F.attention_saliency(q.to(cuda), k.to(cuda))
    assert torch.isfinite(got).all()
    assert abs(got.sum().item() - 4 * 700) < 1e-3 * 4 * 700
    close(got, oracle.attention_saliency(q, k), tol=1e-3)


def test_page_features_vs_oracle(cuda):
    q, k = qk(1000, 1000, 8, 8, 128, 11)
    sal = F.attention_saliency(q.to(cuda), k.to(cuda))
    S, N = F.page_features(k.to(cuda), 16, token_saliency=sal)
    oS, oN = oracle.page_features(k, 16, sal.cpu().numpy())
    close(S, oS)
    close(N, oN)
    assert float(S.max()) == 1.0 and float(S.min()) >= 0.0 and float(N.max()) <= 1.0
    S2, N2 = F.page_inputs(q.to(cuda), k.to(cuda), 16)
    assert torch.equal(S2, S) and torch.equal(N2, N)
    none, N3 = F.page_features(k.to(cuda), 16)
    assert none is None and torch.equal(N3, N)


def test_page_novelty_odd_rows_and_unaligned_pool(cuda):
    """Rows whose length is not a multiple of 8, and a pool starting 2 bytes past a
    16-byte boundary, take the element-wise path; both match the oracle."""
    g = torch.Generator().manual_seed(17)
    k = torch.randn(301, 1, 100, generator=g).to(torch.bfloat16)
    _, N = F.page_features(k.to(cuda), 16)
    close(N, oracle.page_features(k, 16, None)[1])
    base = torch.randn(1 + 257 * 8 * 128, generator=g).to(torch.bfloat16).to(cuda)
    kk = base[1:].view(257, 8, 128)
    _, N2 = F.page_features(kk, 16)
    close(N2, oracle.page_features(kk.cpu(), 16, None)[1])


def test_saliency_repeatable_and_feeds_policy(cuda):
    """Bitwise repeatable; the page inputs run through the GPU score kernel."""
    from ashkv.runtime.score import score_vectorized
    q, k = qk(512, 512, 4, 4, 64, 5)
    a = F.attention_saliency(q.to(cuda), k.to(cuda))
    b = F.attention_saliency(q.to(cuda), k.to(cuda))
    assert torch.equal(a, b)
    S, N = F.page_features(k.to(cuda), 16, token_saliency=a)
    n = S.numel()
    T = np.linspace(0, 1, n, dtype=np.float32)
    P = np.zeros(n, dtype=np.float32)
    R = score_vectorized(T, S.cpu().numpy(), N.cpu().numpy(), P, 0.7, 0.1, 0.1, 0.1)
    want = oracle.score(T, S.cpu().numpy(), N.cpu().numpy(), P, 0.7, 0.1, 0.1, 0.1)
    assert np.array_equal(R, want)
