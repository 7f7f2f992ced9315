"""GPU parity for the FP8 and INT4 codecs (``fp8_default``, ``int4_default``).

FP8: the kernels against the oracle and against torch's own CUDA casts
(``to(torch.float8_e4m3fn)`` and back), which is what the reference's
FP8Codec runs on a GPU -- every bf16 bit pattern and every code, bit-exact.
INT4: the kernels against the reference's own blobs (tests/golden) and the
oracle, over every fast and generic group size, special values, ragged and
unaligned buffers, and a full-size KV tensor.
"""
from __future__ import annotations

import struct

import numpy as np
import pytest
import torch

import oracle
from conftest import GOLDEN

from ashkv import _native
from ashkv.codecs import FP8Codec, INT4Codec
from ashkv.codecs import fp8 as fp8_mod
from ashkv.codecs import int4 as int4_mod

pytestmark = pytest.mark.gpu

F84 = np.load(GOLDEN / "fp8_int4.npz")


def bits_of(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16).reshape(-1)


def dev_bits(bits: np.ndarray, dev) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits, dtype=np.uint16).view(np.int16)).to(dev).view(torch.bfloat16)


# ----------------------------------------------------------------------------- FP8
def test_fp8_encode_every_bf16_pattern(cuda):
    allb = np.arange(65536, dtype=np.uint16)
    x = dev_bits(allb, cuda)
    ours = fp8_mod.encode_tensor(x).cpu().numpy()
    np.testing.assert_array_equal(ours, oracle.fp8_encode(allb))
    torch_cuda = x.to(torch.float8_e4m3fn).view(torch.uint8).cpu().numpy()
    np.testing.assert_array_equal(ours, torch_cuda)
    np.testing.assert_array_equal(ours, F84["fp8_encode_all"])


def test_fp8_decode_every_code(cuda):
    codes = torch.arange(256, dtype=torch.int32).to(torch.uint8).to(cuda)
    ours = bits_of(fp8_mod.decode_tensor(codes))
    np.testing.assert_array_equal(ours, oracle.fp8_decode(np.arange(256, dtype=np.uint8)))
    torch_cuda = bits_of(codes.view(torch.float8_e4m3fn).to(torch.bfloat16))
    np.testing.assert_array_equal(ours, torch_cuda)


@pytest.mark.parametrize("n,offset", [(1, 0), (15, 0), (17, 0), (16 * 1000 + 5, 0), (4099, 1), (64, 3)])
def test_fp8_ragged_and_unaligned(cuda, n, offset):
    rng = np.random.default_rng(n + offset)
    bits = rng.integers(0, 65536, n + offset, dtype=np.uint16)
    x = dev_bits(bits, cuda)[offset:]
    codes = torch.zeros(n + offset, dtype=torch.uint8, device=cuda)[offset:]
    _native.fp8_encode(x, codes)
    np.testing.assert_array_equal(codes.cpu().numpy(), oracle.fp8_encode(bits[offset:]))
    out = torch.zeros(n + offset, dtype=torch.bfloat16, device=cuda)[offset:]
    _native.fp8_decode(codes, out)
    np.testing.assert_array_equal(bits_of(out), oracle.fp8_decode(codes.cpu().numpy()))


def test_fp8_codec_bytes_api(cuda):
    torch.manual_seed(42)
    arr = torch.randn(128, dtype=torch.bfloat16) * 10
    data = arr.view(torch.int16).numpy().tobytes()
    codec = FP8Codec()
    enc = codec.encode(data)
    assert enc == oracle.fp8_encode(np.frombuffer(data, np.uint16)).tobytes()
    dec = codec.decode(enc)
    assert dec == oracle.fp8_decode(np.frombuffer(enc, np.uint8)).tobytes()
    assert codec.encode(b"") == b"" and codec.decode(b"") == b""
    with pytest.raises(ValueError):
        codec.encode(b"\x00\x01\x02")


def test_fp8_full_kv_tensor_matches_torch_cast(cuda):
    """One K tensor of the INT4-dithered workload's shape [4096, 16, 8, 128] (67M elements)."""
    g = torch.Generator(device=cuda).manual_seed(7)
    x = (torch.randn(4096 * 16 * 8 * 128, generator=g, device=cuda) * 64).to(torch.bfloat16)
    ours = fp8_mod.encode_tensor(x)
    assert torch.equal(ours, x.to(torch.float8_e4m3fn).view(torch.uint8))
    back = fp8_mod.decode_tensor(ours)
    assert torch.equal(back.view(torch.int16), ours.view(torch.float8_e4m3fn).to(torch.bfloat16).view(torch.int16))


# ----------------------------------------------------------------------------- INT4
@pytest.mark.parametrize("ci", range(len(F84["int4_group_size"])))
def test_int4_codec_matches_reference_blob(cuda, ci):
    gs = int(F84["int4_group_size"][ci])
    codec = INT4Codec(group_size=gs)
    data = F84[f"int4_in_{ci}"].tobytes()
    blob = codec.encode(data)
    assert blob == F84[f"int4_blob_{ci}"].tobytes()
    assert codec.decode(blob) == F84[f"int4_dec_{ci}"].tobytes()


def test_int4_decode_random_reference_blob(cuda):
    blob = F84["int4_rand_blob"].tobytes()
    n_groups, n_values = struct.unpack("<II", blob[:8])
    assert INT4Codec(group_size=n_values // n_groups).decode(blob) == F84["int4_rand_dec"].tobytes()


def test_int4_empty_and_malformed(cuda):
    codec = INT4Codec()
    assert codec.encode(b"") == F84["int4_empty_blob"].tobytes()
    assert codec.decode(codec.encode(b"")) == b""
    assert codec.decode(struct.pack("<II", 0, 0)) == b""
    with pytest.raises(ValueError):   # num_values inconsistent with the codec's group size
        codec.decode(struct.pack("<II", 1, 32) + b"\x00\x3f" + bytes(16))
    with pytest.raises(ValueError):   # 7 groups of 7 values: odd padded count
        INT4Codec(group_size=7).encode(bytes(2 * 49))


def _wide_groups(n: int, gs: int, seed: int) -> np.ndarray:
    """N(0,1) values with a per-group scale spanning 1e-12 .. 1e32, plus zeros and ties."""
    g = torch.Generator().manual_seed(seed)
    n_groups = -(-n // gs)
    scale = torch.exp(torch.empty(n_groups).uniform_(-27.0, 73.0, generator=g))
    x = torch.randn(n_groups * gs, generator=g) * scale.repeat_interleave(gs)
    x[torch.randperm(x.numel(), generator=g)[: x.numel() // 50]] = 0.0
    return x[:n].to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16).copy()


@pytest.mark.parametrize("gs", [8, 16, 32, 64, 128, 256, 24, 48, 96, 512, 7, 1, 2, 1000])
def test_int4_group_sizes_vs_oracle(cuda, gs):
    n = gs * 300 - (gs // 3) * 2        # 300 groups (even padded count), the last one ragged
    bits = _wide_groups(n, gs, gs)
    sc_o, pk_o, total = oracle.int4_encode(bits, gs)
    scales, packed, total_k = int4_mod.encode_tensor(dev_bits(bits, cuda), gs)
    assert total_k == total
    np.testing.assert_array_equal(bits_of(scales), sc_o)
    np.testing.assert_array_equal(packed.cpu().numpy(), pk_o)
    out = int4_mod.decode_tensor(scales, packed, gs)
    np.testing.assert_array_equal(bits_of(out), oracle.int4_decode(sc_o, pk_o, gs))


@pytest.mark.parametrize("gs", [16, 32, 64, 256])
def test_int4_every_quotient_of_a_binade(cuda, gs):
    """Groups that start with each bf16 absmax in [1, 2) and walk every bf16 value of
    magnitude <= it (both signs): every quotient 7x / am the encoder can form."""
    groups = []
    for a in range(0x3F80, 0x4000):
        mags = np.arange(0, a + 1, dtype=np.uint32)
        vals = np.concatenate([mags, mags | 0x8000]).astype(np.uint16)
        vals = np.concatenate([vals, np.zeros((-len(vals)) % (gs - 1), np.uint16)]).reshape(-1, gs - 1)
        groups.append(np.concatenate([np.full((len(vals), 1), a, np.uint16), vals], axis=1))
    bits = np.concatenate(groups).reshape(-1)
    if (bits.size // gs) % 2:
        bits = np.concatenate([bits, np.zeros(gs, np.uint16)])
    sc_o, pk_o, _ = oracle.int4_encode(bits, gs)
    scales, packed, _ = int4_mod.encode_tensor(dev_bits(bits, cuda), gs)
    np.testing.assert_array_equal(bits_of(scales), sc_o)
    np.testing.assert_array_equal(packed.cpu().numpy(), pk_o)


def test_int4_decode_every_nibble_and_scale(cuda):
    """All 16 nibbles under every bf16 scale pattern."""
    sc = np.arange(65536, dtype=np.uint16)
    pk = np.tile(np.array([0x01, 0x23, 0x45, 0x67, 0x89, 0xAB, 0xCD, 0xEF], np.uint8), 65536)
    out = int4_mod.decode_tensor(dev_bits(sc, cuda), torch.from_numpy(pk).to(cuda), 16)
    np.testing.assert_array_equal(bits_of(out), oracle.int4_decode(sc, pk, 16))


@pytest.mark.parametrize("gs", [64, 16])
def test_int4_unaligned_buffers(cuda, gs):
    n = gs * 97
    bits = _wide_groups(n + 1, gs, 5)[1:]
    x = dev_bits(np.concatenate([[0], bits]).astype(np.uint16), cuda)[1:]   # 2-byte aligned
    sc_o, pk_o, total = oracle.int4_encode(bits, gs)
    n_groups = total // gs
    scales = torch.empty(n_groups, dtype=torch.bfloat16, device=cuda)
    packed = torch.empty(total // 2 + 1, dtype=torch.uint8, device=cuda)[1:]   # odd address
    _native.int4_encode(x, gs, scales, packed)
    np.testing.assert_array_equal(bits_of(scales), sc_o)
    np.testing.assert_array_equal(packed.cpu().numpy(), pk_o)
    out = torch.empty(total + 1, dtype=torch.bfloat16, device=cuda)[1:]
    _native.int4_decode(scales, packed, n_groups, gs, out)
    np.testing.assert_array_equal(bits_of(out), oracle.int4_decode(sc_o, pk_o, gs))


def test_int4_random_scales_decode_vs_oracle(cuda):
    """Decode arithmetic over the whole bf16 scale range (subnormal, huge, inf, NaN, negative)."""
    rng = np.random.default_rng(11)
    for gs in (64, 16, 8, 24):
        n_groups = 4096
        sc = rng.integers(0, 65536, n_groups, dtype=np.uint16)
        pk = rng.integers(0, 256, n_groups * gs // 2, dtype=np.uint8)
        out = int4_mod.decode_tensor(dev_bits(sc, cuda), torch.from_numpy(pk).to(cuda), gs)
        np.testing.assert_array_equal(bits_of(out), oracle.int4_decode(sc, pk, gs))


def test_int4_full_kv_tensor_vs_oracle(cuda):
    """One K tensor [4096, 16, 8, 128] (67M elements), default group size 64."""
    g = torch.Generator().manual_seed(3)
    x = torch.randn(4096 * 16 * 8 * 128, generator=g)
    x[torch.randint(0, x.numel(), (x.numel() // 1000,), generator=g)] *= 50
    bits = x.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    scales, packed, total = int4_mod.encode_tensor(dev_bits(bits, cuda), 64)
    sc_o, pk_o, _ = oracle.int4_encode(bits, 64)
    np.testing.assert_array_equal(bits_of(scales), sc_o)
    np.testing.assert_array_equal(packed.cpu().numpy(), pk_o)
    out = int4_mod.decode_tensor(scales, packed, 64)
    np.testing.assert_array_equal(bits_of(out), oracle.int4_decode(sc_o, pk_o, 64))
