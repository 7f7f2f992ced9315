"""Quality of the production dither against the reference's kind of dither.

The reference dithers with ``torch.rand`` (fp32 uniforms, 24 random bits);
this library's production path draws centred 8-bit uniforms, U = (b + 0.5) / 256,
from an in-kernel Philox4x32-10 stream.  The reference's adversarial stress test
(ashkv/tests/stress_test_nbit.py:50-89: 1024 tokens x 8 heads x 64, K and V
N(0, 0.02^2) with 1 % of the entries shifted by 50 standard deviations, the
attention output of decoded K/V against the original, thresholds INT2 > 0.98,
INT4 > 0.999, INT8 > 0.9999) is rebuilt here with seeded inputs and run both
ways: the Philox path must pass the reference's thresholds and stay within a
small margin of the same codec given fp32 ``torch.rand`` uniforms.
"""
from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from ashkv.codecs import DitheredNBitCodec

pytestmark = pytest.mark.gpu

THRESHOLDS = {2: 0.98, 4: 0.999, 8: 0.9999}


def adversarial(shape, gen, dev) -> torch.Tensor:
    x = (torch.randn(shape, generator=gen, device=dev) * 0.02).to(torch.bfloat16)
    flat = x.view(-1)
    n_out = flat.numel() // 100
    idx = torch.randperm(flat.numel(), generator=gen, device=dev)[:n_out]
    sign = torch.randint(0, 2, (n_out,), generator=gen, device=dev).float() * 2 - 1
    flat[idx] += (sign * 50.0 * flat.float().std()).to(torch.bfloat16)
    return x


def attn_cosine(q, k, v, k2, v2) -> float:
    a = F.scaled_dot_product_attention(q.transpose(0, 1), k.transpose(0, 1), v.transpose(0, 1))
    b = F.scaled_dot_product_attention(q.transpose(0, 1), k2.transpose(0, 1), v2.transpose(0, 1))
    return F.cosine_similarity(a.float().reshape(-1), b.float().reshape(-1), dim=0).item()


def roundtrip(codec, x: torch.Tensor, uniform=None) -> torch.Tensor:
    raw = x.contiguous().view(torch.int16).cpu().numpy().tobytes()
    out = codec.decode(codec.encode(raw, uniform=uniform))
    return torch.frombuffer(bytearray(out), dtype=torch.bfloat16).to(x.device).view_as(x)


@pytest.mark.parametrize("bits", [2, 4, 8])
def test_production_dither_matches_fp32_uniform_quality(cuda, bits):
    gen = torch.Generator(device=cuda).manual_seed(42)
    S, H, D = 1024, 8, 64
    k, v = adversarial((S, H, D), gen, cuda), adversarial((S, H, D), gen, cuda)
    q = (torch.randn((S, H, D), generator=gen, device=cuda) * 0.02).to(torch.bfloat16)
    cos_philox = attn_cosine(q, k, v, roundtrip(DitheredNBitCodec(hidden_dim=D, bits=bits), k),
                             roundtrip(DitheredNBitCodec(hidden_dim=D, bits=bits), v))
    ug = torch.Generator(device=cuda).manual_seed(7)
    uk = torch.rand(k.numel(), generator=ug, device=cuda)
    uv = torch.rand(v.numel(), generator=ug, device=cuda)
    cos_fp32 = attn_cosine(q, k, v, roundtrip(DitheredNBitCodec(hidden_dim=D, bits=bits), k, uk),
                           roundtrip(DitheredNBitCodec(hidden_dim=D, bits=bits), v, uv))
    assert cos_philox > THRESHOLDS[bits], (bits, cos_philox)
    assert cos_fp32 > THRESHOLDS[bits], (bits, cos_fp32)
    # the 8-bit uniforms cost at most a sliver of the fp32 uniforms' fidelity
    assert (1.0 - cos_philox) <= 1.5 * (1.0 - cos_fp32) + 1e-6, (bits, cos_philox, cos_fp32)
