"""GPU parity: the sm_100a codec kernels (through the C ABI) against the oracle.

Integer/byte outputs (codes, scales, outlier lists, packed blobs, decoded
bf16 bits) must be bit-exact, with one exception: INT8 codes may be one apart
from the oracle's at tie-zone elements (the reference divides with the GPU's
approximate div.full.f32, which this library reproduces and the CPU oracle
cannot; see ``conftest.assert_int8_codes``).  The oracle itself is pinned to
the reference's outputs by tests/test_oracle_golden.py, and the kernels are
compared with the reference's own B200 outputs, exactly, by
tests/test_gpu_reference_fixtures.py.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from conftest import GOLDEN, assert_int8_codes

from ashkv import _native
from ashkv.codecs import DitheredINT2Codec, DitheredNBitCodec, INT8Codec
from ashkv.codecs import int8 as int8_mod
from ashkv.codecs import nbit_dithered as nb

pytestmark = pytest.mark.gpu

NBIT = np.load(GOLDEN / "nbit.npz")
INT8 = np.load(GOLDEN / "int8.npz")


def bits_of(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16).reshape(-1)


def rand_bf16(n: int, seed: int, kind: str = "normal") -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(n, generator=g)
    if kind == "wide":
        x = x * torch.exp(torch.randn(n, generator=g) * 3.0)
    elif kind == "outliers":
        pos = torch.randperm(n, generator=g)[: max(1, n // 1000)]
        x[pos] *= 50.0
    return x.to(torch.bfloat16)


# ------------------------------------------------------------------- INT8
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("row_len", [128, 1024, 4096, 8, 16, 24, 32, 64, 136, 256, 512, 2048])
@pytest.mark.parametrize("fp32_product", [False, True])
def test_int8_rows_bitexact(cuda, dtype, row_len, fp32_product):
    n_rows = 300
    x = (rand_bf16(n_rows * row_len, row_len, "wide").float() * 0.25).to(dtype).view(n_rows, row_len)
    codes = torch.empty(n_rows, row_len, dtype=torch.int8, device=cuda)
    scales = torch.empty(n_rows, dtype=dtype, device=cuda)
    _native.int8_encode_rows(x.to(cuda), codes, scales, fp32_product=fp32_product)
    oc, osc, tie = oracle.int8_encode(bits_of(x), row_len, src_fp16=dtype == torch.float16,
                                      scale_fp16=dtype == torch.float16, fp32_product=fp32_product, with_ties=True)
    got = codes.cpu().numpy()
    assert_int8_codes(got, oc, tie)
    assert np.array_equal(bits_of(scales), osc)
    for out_dtype in (torch.bfloat16, torch.float16):
        dec = torch.empty(n_rows, row_len, dtype=out_dtype, device=cuda)
        _native.int8_decode_rows(codes, scales, dec)
        want = oracle.int8_decode(got, osc, scale_fp16=dtype == torch.float16, dst_fp16=out_dtype == torch.float16)
        assert np.array_equal(bits_of(dec), want.reshape(-1))


def rows_under_absmax(L: int, am_bits, fill_tiny: bool = False) -> np.ndarray:
    """bf16 rows of length L: for each absmax pattern a, rows that start with a and
    then walk every bf16 pattern of magnitude <= a, both signs, so every quotient
    s / am an encoder can form for that absmax occurs."""
    rows = []
    for a in am_bits:
        mags = np.arange(0, int(a) + 1, dtype=np.uint32)
        vals = np.concatenate([mags, mags | 0x8000]).astype(np.uint16)
        pad = (-len(vals)) % (L - 1)
        vals = np.concatenate([vals, np.zeros(pad, np.uint16)]).reshape(-1, L - 1)
        rows.append(np.concatenate([np.full((len(vals), 1), a, np.uint16), vals], axis=1))
    return np.concatenate(rows)


@pytest.mark.parametrize("L", [128, 1024])
def test_int8_rows_every_quotient_of_a_binade(cuda, L):
    """Every bf16 absmax in [1, 2) (the quotient's rounding is invariant under
    power-of-two scaling of both operands) against every bf16 value below it, plus
    zero rows, rows under the 1e-8 floor and rows at the extremes of the range."""
    am = list(range(0x3F80, 0x4000)) + [0x0001, 0x0080, 0x2000, 0x3300, 0x7F7F]
    bits = rows_under_absmax(L, am)
    extra = np.zeros((4, L), np.uint16)
    extra[1, :] = 0x3100        # 1.86e-9: every row value under the 1e-8 floor
    extra[2, ::3] = 0x8001      # negative subnormals
    extra[3, :] = 0x7F80        # +inf
    bits = np.concatenate([bits, extra])
    x = torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).to(cuda)
    for sdt in (torch.bfloat16, torch.float16):
        codes, scales = int8_mod.encode_rows(x, scale_dtype=sdt)
        oc, osc, tie = oracle.int8_encode(bits, L, scale_fp16=sdt == torch.float16, with_ties=True)
        n_ties = assert_int8_codes(codes.cpu().numpy(), oc, tie)
        assert n_ties <= 0.001 * oc.size, n_ties
        assert np.array_equal(bits_of(scales), osc)


@pytest.mark.parametrize("sdt", [torch.bfloat16, torch.float16])
def test_int8_decode_every_code_and_scale(cuda, sdt):
    """All 256 codes under every 16-bit scale pattern (subnormal, huge, inf, NaN, negative)."""
    codes = np.tile(np.arange(-128, 128, dtype=np.int8), (65536, 1))
    sc = np.arange(65536, dtype=np.uint16)
    out = int8_mod.decode_rows(torch.from_numpy(codes).to(cuda),
                               torch.from_numpy(sc.view(np.int16)).view(sdt).to(cuda))
    want = oracle.int8_decode(codes, sc, scale_fp16=sdt == torch.float16)
    assert np.array_equal(bits_of(out), want.reshape(-1))


@pytest.mark.parametrize("ci", range(int(INT8["int8_n_cases"])))
def test_int8_kernel_matches_reference_golden(cuda, ci):
    pre = f"int8_{ci}_"
    rows, L, _ = (int(v) for v in INT8[pre + "meta"])
    src = torch.from_numpy(INT8[pre + "src"].view(np.int16).copy()).view(torch.float16).view(rows, L)
    codes = torch.empty(rows, L, dtype=torch.int8, device=cuda)
    scales = torch.empty(rows, dtype=torch.float16, device=cuda)
    _native.int8_encode_rows(src.to(cuda), codes, scales)
    got = codes.cpu().numpy()
    x = src.float().numpy()
    # fp16 product is inf: the interpreter's cast of that differs from the GPU's
    overflow = np.abs(x) * 127.0 > 65504.0
    # the interpreter divides exactly, the GPU kernel as Triton does on the device
    _, _, tie = oracle.int8_encode(INT8[pre + "src"], L, src_fp16=True, scale_fp16=True, with_ties=True)
    assert_int8_codes(got[~overflow], INT8[pre + "codes"][~overflow], tie[~overflow])
    assert np.array_equal(bits_of(scales), INT8[pre + "scales"])


def test_int8_gather_and_flat_scale_slots(cuda):
    """Hook layout: rows gathered by index, codes into slot rows, fp16 scales at the
    reference's flat positions (token t -> slot t // H, offset 2 * (t % H))."""
    H, D, n, cap = 8, 128, 37, 100
    L = H * D
    pool = rand_bf16(cap * L, 3).view(cap, L).to(cuda)
    idx = torch.randperm(cap, generator=torch.Generator().manual_seed(4))[:n].to(cuda)
    slot = 2 * H * D
    staging = torch.zeros(n, slot, dtype=torch.uint8, device=cuda)
    codes_view = staging[:, 2 * H:2 * H + L].view(torch.int8)
    scales_base = staging.view(-1)[:].view(torch.float16)  # scale t at byte (t//H)*slot + 2*(t%H)
    _native.int8_encode_rows(pool, codes_view, scales_base, row_index=idx, scales_per_slot=H,
                             scale_slot_stride=slot)
    oc, osc, tie = oracle.int8_encode(bits_of(pool[idx.cpu()]), L, scale_fp16=True, with_ties=True)
    st = staging.cpu().numpy()
    got = st[:, 2 * H:2 * H + L].view(np.int8)
    assert_int8_codes(got, oc, tie)
    flat = st[:, :2 * H].copy().view(np.uint16).reshape(-1)  # concatenated per-slot scale regions
    assert np.array_equal(flat[:n], osc)
    # decode straight back into a scattered destination
    out = torch.zeros(cap, L, dtype=torch.bfloat16, device=cuda)
    _native.int8_decode_rows(codes_view, scales_base, out, row_index=idx, scales_per_slot=H, scale_slot_stride=slot)
    want = oracle.int8_decode(got, osc, scale_fp16=True)
    assert np.array_equal(bits_of(out[idx]).reshape(n, L), want)


def test_int8_codec_bytes_api_matches_oracle(cuda):
    x = rand_bf16(123 * 128 + 5, 9)  # ragged tail: trailing values are dropped
    codec = INT8Codec()
    blob = codec.encode(bits_of(x).tobytes())
    oc, osc, tie = oracle.int8_encode(bits_of(x)[:123 * 128], 128, with_ties=True)
    assert blob[:4 + 2 * 123] == oracle.int8_blob(oc, osc)[:4 + 2 * 123] and len(blob) == 4 + 123 * 130
    got = np.frombuffer(blob, np.int8, 123 * 128, 4 + 2 * 123).reshape(123, 128)
    assert_int8_codes(got, oc, tie)
    dec = codec.decode(blob)
    assert dec == oracle.int8_decode(got, osc).tobytes()
    assert codec.encode(b"") == b"\x00\x00\x00\x00"
    assert codec.encode(b"\x00\x01" * 10) == b"\x00\x00\x00\x00"
    assert codec.decode(b"\x00\x00\x00\x00") == b"" and codec.decode(b"\x01") == b""
    with pytest.raises(ValueError):
        codec.encode(b"\x00\x01\x02")


def test_int8_reference_fidelity_budget(cuda):
    """The reference GPU test's bounds: cos > 0.99, MSE < 0.05 on fp16 [1024, 32, 128]."""
    g = torch.Generator(device="cpu").manual_seed(0)
    x = (torch.randn(1024, 32, 128, generator=g) * 0.5 + 0.1).half().to(cuda)
    codes, scales = int8_mod.encode_rows(x.view(1024, -1), scale_dtype=torch.float16)
    y = int8_mod.decode_rows(codes, scales, out_dtype=torch.float16)
    a, b = x.float().view(-1), y.float().view(-1)
    assert torch.nn.functional.cosine_similarity(a[None], b[None]).item() > 0.99
    assert torch.nn.functional.mse_loss(a, b).item() < 0.05


def test_int8_nan_inf_do_not_crash(cuda):
    x = torch.zeros(2, 1, 128, dtype=torch.float16, device=cuda)
    x[0, 0, 0], x[0, 0, 1], x[1, 0, 0] = float("inf"), float("nan"), 65504.0
    codes, scales = int8_mod.encode_rows(x.view(2, -1), scale_dtype=torch.float16)
    torch.cuda.synchronize()
    assert codes.shape == (2, 128)
    c = codes.cpu()
    assert c[0, 1].item() == 0  # NaN -> 0


@pytest.mark.parametrize("L", [128, 1024, 32])
def test_int8_rows_with_nan_and_inf_match_oracle(cuda, L):
    """NaN is ignored by the row maximum (and codes 0); a row whose absmax is
    infinite divides with div.full.f32 (every finite value gives 0); an all-NaN
    row falls to the 1e-8 floor."""
    g = torch.Generator().manual_seed(5)
    x = torch.randn(64, L, generator=g).to(torch.bfloat16)
    b = x.view(torch.int16).numpy().view(np.uint16).copy()
    b[0, 0] = 0x7FC0                # NaN in the first lane's first chunk
    b[1, L - 1] = 0xFFC1            # negative NaN with a payload, last element
    b[2, 3], b[2, 5] = 0x7F80, 0x7FC0
    b[3, :] = 0x7FC0                # every element NaN
    b[4, L // 2] = 0xFF80           # -inf
    b[5, ::2] = 0x7FA0              # signalling-NaN pattern on every other element
    b[6, :] = 0
    xb = torch.from_numpy(b.view(np.int16)).view(torch.bfloat16).to(cuda)
    for sdt in (torch.bfloat16, torch.float16):
        codes, scales = int8_mod.encode_rows(xb, scale_dtype=sdt)
        oc, osc, tie = oracle.int8_encode(b, L, scale_fp16=sdt == torch.float16, with_ties=True)
        assert_int8_codes(codes.cpu().numpy(), oc, tie)
        assert np.array_equal(bits_of(scales), osc)


# ------------------------------------------------------------------- N-bit
@pytest.mark.parametrize("ci", range(int(NBIT["nbit_n_cases"])))
def test_nbit_bytes_api_reproduces_reference_blob(cuda, ci):
    pre = f"nbit_{ci}_"
    bits, hidden, is_int2, n, _trail = (int(v) for v in NBIT[pre + "meta"])
    sigma = float(NBIT[pre + "sigma"])
    codec = DitheredINT2Codec(hidden) if is_int2 else DitheredNBitCodec(hidden, 32, sigma, bits)
    src = NBIT[pre + "src"].tobytes()
    blob = codec.encode(src, uniform=NBIT[pre + "u"] if n else None)
    assert blob == NBIT[pre + "blob"].tobytes()
    assert codec.decode(blob) == NBIT[pre + "decoded"].tobytes()


@pytest.mark.parametrize("bits", [2, 4, 8])
@pytest.mark.parametrize("kind", ["normal", "wide", "outliers"])
def test_nbit_kernel_vs_oracle_tensor_dither(cuda, bits, kind):
    n = 300 * 8192 + 96  # ragged last bucket
    x = rand_bf16(n, 17 + bits, kind)
    u = torch.rand(n, generator=torch.Generator().manual_seed(5))
    enc = nb.encode_groups(x.to(cuda), bits, 3.0, uniform=u.to(cuda))
    osc, ocodes, oidx, ovals = oracle.nbit_encode(bits_of(x), bits, u.numpy(), 3.0)
    assert np.array_equal(bits_of(enc.scales), osc)
    assert np.array_equal(enc.codes[: ocodes.size].cpu().numpy(), ocodes)
    idx, val, total = nb.flatten_outliers(enc)
    t = int(total.item())
    assert t == oidx.size
    assert np.array_equal(idx[:t].cpu().numpy(), oidx)
    assert np.array_equal(val[:t].cpu().numpy().view(np.uint16), ovals)
    assert int(enc.status.item()) == 0
    dec = nb.decode_groups(enc)
    want = oracle.nbit_decode(osc, ocodes, bits, oidx, ovals)
    assert np.array_equal(bits_of(dec), want)


def _offset_and_threshold_groups(n_groups: int, seed: int) -> np.ndarray:
    """Groups whose mean dwarfs their spread (offsets up to 1e5 sd, both signs),
    groups of bf16-quantised offsets (many equal values), and groups with one
    element moved to about 3 sd from the rest, to sit near the outlier threshold."""
    g = torch.Generator().manual_seed(seed)
    z = torch.randn(n_groups, 32, generator=g)
    offs = torch.tensor([0.0, 3.0, 30.0, 300.0, 3e3, 3e4, 1e5, -1e5, -7.0])
    k = torch.randint(0, offs.numel(), (n_groups, 1), generator=g)
    sd = torch.exp(torch.empty(n_groups, 1).uniform_(-8.0, 8.0, generator=g))
    x = (offs[k] + z) * sd
    near = torch.rand(n_groups, generator=g) < 0.25
    mult = torch.empty(n_groups).uniform_(2.9, 3.3, generator=g)
    x[near, 0] = (offs[k[near, 0]] + mult[near] * 1.0) * sd[near, 0]
    return x.reshape(-1).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16).copy()


@pytest.mark.parametrize("bits", [4, 2])
def test_nbit_offset_and_near_threshold_groups_vs_oracle(cuda, bits):
    n_groups = 1 << 16
    xb = _offset_and_threshold_groups(n_groups, 99 + bits)
    n = xb.size
    u = torch.rand(n, generator=torch.Generator().manual_seed(6))
    x = torch.from_numpy(xb.view(np.int16)).view(torch.bfloat16)
    enc = nb.encode_groups(x.to(cuda), bits, 3.0, uniform=u.to(cuda))
    osc, ocodes, oidx, ovals = oracle.nbit_encode(xb, bits, u.numpy(), 3.0)
    assert oidx.size > n_groups // 50  # the near-threshold elements produce outliers
    assert np.array_equal(bits_of(enc.scales), osc)
    assert np.array_equal(enc.codes[: ocodes.size].cpu().numpy(), ocodes)
    idx, val, total = nb.flatten_outliers(enc)
    t = int(total.item())
    assert t == oidx.size and np.array_equal(idx[:t].cpu().numpy(), oidx)
    assert np.array_equal(val[:t].cpu().numpy().view(np.uint16), ovals)


@pytest.mark.parametrize("bits", [2, 4])
def test_nbit_philox_dither_matches_oracle(cuda, bits):
    n = 64 * 8192
    x = rand_bf16(n, 23, "outliers")
    seed, offset = 0x1234_5678_9ABC, 4096
    enc = nb.encode_groups(x.to(cuda), bits, 3.0, seed=seed, dither_offset=offset)
    u = oracle.philox_dither(n, seed, offset)
    osc, ocodes, oidx, ovals = oracle.nbit_encode(bits_of(x), bits, u, 3.0)
    assert np.array_equal(bits_of(enc.scales), osc)
    assert np.array_equal(enc.codes[: ocodes.size].cpu().numpy(), ocodes)


# A group of INT4-grid values (multiples of 2.8027344 / 7 rounded to bf16, largest 2.0) and
# 8-bit-grid uniforms: element 5 lands one ulp above a rounding tie, v = RN(RN(a / delta) + 1.5)
# = 0.5 + 2^-24, and only a separately rounded noise term a = RN(x + RN((U - 0.5) * delta))
# gives code 1 there (a fused x + (U - 0.5) * delta gives 0).
NEAR_TIE_X = [0.80078125, 0.0, 0.80078125, -1.1953125, 1.6015625, -1.6015625, -1.1953125, 2.0,
              -0.80078125, 0.80078125, -0.400390625, 0.400390625, 0.400390625, 1.1953125, 0.400390625,
              -1.1953125, 2.0, 1.6015625, -0.80078125, -0.400390625, -0.80078125, 1.6015625, -0.80078125,
              0.80078125, 0.400390625, -0.400390625, 0.0, 0.80078125, -0.400390625, 1.6015625, 0.0, 0.0]
NEAR_TIE_B = [242, 149, 154, 8, 145, 179, 65, 14, 215, 95, 213, 12, 145, 82, 73, 105,
              224, 194, 174, 12, 116, 164, 7, 17, 218, 86, 20, 168, 152, 51, 7, 183]


@pytest.mark.parametrize("bits", [2, 4, 8])
def test_nbit_noise_rounded_separately(cuda, bits):
    x = torch.tensor(NEAR_TIE_X * 32, dtype=torch.float32).to(torch.bfloat16)
    u = ((torch.tensor(NEAR_TIE_B * 32, dtype=torch.float32) + 0.5) / 256.0)
    enc = nb.encode_groups(x.to(cuda), bits, 3.0, uniform=u.to(cuda))
    osc, ocodes, _, _ = oracle.nbit_encode(bits_of(x), bits, u.numpy(), 3.0)
    assert np.array_equal(bits_of(enc.scales), osc)
    assert np.array_equal(enc.codes[: ocodes.size].cpu().numpy(), ocodes)
    if bits == 2:
        assert (int(ocodes[1]) >> 4) & 3 == 1  # the near-tie element


@pytest.mark.parametrize("bits", [2, 4, 8])
@pytest.mark.parametrize("mode", ["tensor", "philox"])
def test_nbit_structured_values_match_oracle(cuda, bits, mode):
    """INT4-decoded values (a small grid per 64 elements) with uniforms on the 8-bit
    grid hit exact and one-ulp rounding ties of the quantiser far more often than
    Gaussian data does; every code, delta and outlier must still equal the oracle's."""
    n = 32 * 32768
    x = rand_bf16(n, 91, "outliers")
    sc, pk, _ = oracle.int4_encode(bits_of(x), 64)
    xs = oracle.int4_decode(sc, pk, 64)[:n]
    xt = torch.from_numpy(xs.view(np.int16).copy()).view(torch.bfloat16)
    if mode == "tensor":
        g = torch.Generator().manual_seed(bits)
        u = (torch.randint(0, 256, (n,), generator=g).float() + 0.5) / 256.0
        enc = nb.encode_groups(xt.to(cuda), bits, 3.0, uniform=u.to(cuda))
        un = u.numpy()
    else:
        enc = nb.encode_groups(xt.to(cuda), bits, 3.0, seed=1234, dither_offset=32768)
        un = oracle.philox_dither(n, 1234, 32768)
    osc, ocodes, oidx, ovals = oracle.nbit_encode(xs, bits, un, 3.0)
    assert np.array_equal(bits_of(enc.scales), osc)
    assert np.array_equal(enc.codes[: ocodes.size].cpu().numpy(), ocodes)
    idx, val, total = nb.flatten_outliers(enc)
    t = int(total.item())
    assert t == oidx.size and np.array_equal(idx[:t].cpu().numpy(), oidx)
    assert np.array_equal(val[:t].cpu().numpy().view(np.uint16), ovals)


def test_nbit_flatten_spans_scan_tiles(cuda):
    """More buckets than one scan tile (4096): flat list and offsets against the oracle."""
    n = 5 * 4096 * 1024 + 32 * 77
    x = rand_bf16(n, 61, "outliers")
    u = torch.rand(n, generator=torch.Generator().manual_seed(8))
    enc = nb.encode_groups(x.to(cuda), 4, 3.0, uniform=u.to(cuda))
    _, _, oidx, ovals = oracle.nbit_encode(bits_of(x), 4, u.numpy(), 3.0)
    nbk = enc.n_buckets
    assert nbk > 4 * 4096
    offsets = torch.empty(_native.nbit_flatten_scratch_ints(nbk), dtype=torch.int32, device=cuda)
    idx = torch.empty(nbk * enc.bucket_cap, dtype=torch.int32, device=cuda)
    val = torch.empty(nbk * enc.bucket_cap, dtype=torch.int16, device=cuda)
    total = torch.empty(1, dtype=torch.int32, device=cuda)
    _native.nbit_outliers_flatten(enc.bucket_counts, enc.bucket_entries, enc.bucket_cap, nbk, offsets, idx, val,
                                  total)
    t = int(total.item())
    assert t == oidx.size
    assert np.array_equal(idx[:t].cpu().numpy(), oidx)
    assert np.array_equal(val[:t].cpu().numpy().view(np.uint16), ovals)
    counts = enc.bucket_counts[:nbk].cpu().numpy().astype(np.int64)
    want = np.concatenate([[0], np.cumsum(counts)])
    assert np.array_equal(offsets[: nbk + 1].cpu().numpy(), want)


def test_nbit_bucket_overflow_is_flagged(cuda):
    n = 4 * 8192
    x = rand_bf16(n, 31, "outliers")
    enc = nb.encode_groups(x.to(cuda), 4, 3.0, uniform=torch.rand(n).to(cuda), bucket_cap=2)
    torch.cuda.synchronize()
    assert int(enc.status.item()) & _native.FLAG_OUTLIER_OVERFLOW
    counts = enc.bucket_counts.cpu().numpy()
    assert counts.max() > 2  # true counts are reported even past the capacity


def test_nbit_decode_paths_agree(cuda):
    n = 40 * 8192
    x = rand_bf16(n, 41, "outliers").to(cuda)
    enc = nb.encode_groups(x, 4, 3.0)
    a = nb.decode_groups(enc)
    idx, val, total = nb.flatten_outliers(enc)
    t = int(total.item())
    b = torch.empty_like(a)
    _native.nbit_decode_flat(enc.scales, enc.codes, enc.n_groups, 4, idx[:t], val[:t], t, b, enc.status)
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))
    # outliers come back exactly
    xi = x.view(-1)[idx[:t].long()]
    assert torch.equal(xi.view(torch.int16), a[idx[:t].long()].view(torch.int16))


def test_nbit_config2_full_size_properties(cuda):
    """The INT4 codec workload (K: [4096, 16, 8, 128], 0.1% x50 outliers) at full size:
    outliers restored bit-exactly, inlier error bounded by one quantisation step,
    and a 1/64 sample of buckets bit-exact against the oracle."""
    n = 4096 * 16 * 8 * 128
    g = torch.Generator(device=cuda).manual_seed(0)
    x = torch.randn(n, generator=g, device=cuda)
    pos = torch.randperm(n, generator=g, device=cuda)[: n // 1000]
    x[pos] *= 50.0
    x = x.to(torch.bfloat16)
    enc = nb.encode_groups(x, 4, 3.0, seed=42)
    dec = nb.decode_groups(enc)
    idx, val, total = nb.flatten_outliers(enc)
    t = int(total.item())
    assert t >= n // 1000  # every injected x50 outlier is beyond 3 sigma of its group
    ii = idx[:t].long()
    assert torch.equal(dec[ii].view(torch.int16), x[ii].view(torch.int16))
    delta = enc.scales.float().repeat_interleave(32)
    err = (dec.float() - x.float()).abs()
    mask = torch.ones(n, dtype=torch.bool, device=cuda)
    mask[ii] = False
    assert bool((err[mask] <= delta[mask] * 1.05).all())
    # sampled bit-exactness against the oracle (same Philox dither)
    xs = bits_of(x)
    sc, codes = bits_of(enc.scales), enc.codes.cpu().numpy()
    for b in range(0, n // 8192, 64):
        lo = b * 8192
        u = oracle.philox_dither(8192, 42, lo)
        osc, ocodes, _, _ = oracle.nbit_encode(xs[lo:lo + 8192], 4, u, 3.0)
        assert np.array_equal(sc[lo // 32:(lo + 8192) // 32], osc)
        assert np.array_equal(codes[lo // 2:(lo + 8192) // 2], ocodes)


@pytest.mark.parametrize("bits,hidden", [(4, 128), (2, 128), (8, 64), (4, 32)])
def test_nbit_pinned_api_matches_bytes_api(cuda, bits, hidden):
    x = rand_bf16(257 * hidden, 71, "outliers")
    data = bits_of(x).tobytes()
    a, b = DitheredNBitCodec(hidden_dim=hidden, bits=bits), DitheredNBitCodec(hidden_dim=hidden, bits=bits)
    for _ in range(2):  # the second call checks the per-call seed stays in step
        blob = a.encode(data)
        pblob = b.encode_pinned(x.view(torch.int16).pin_memory())
        assert pblob.numpy().tobytes() == blob
        out = torch.empty(x.numel() + 8, dtype=torch.bfloat16, pin_memory=True)
        dec = b.decode_pinned(pblob, out)
        assert dec.view(torch.int16).numpy().tobytes() == a.decode(blob)
    # batched calls: the same blobs and seeds as the same calls made one by one
    y = rand_bf16(190 * hidden, 72, "wide")
    seq, bat = DitheredNBitCodec(hidden_dim=hidden, bits=bits), DitheredNBitCodec(hidden_dim=hidden, bits=bits)
    want = [seq.encode(bits_of(t).tobytes()) for t in (x, y, x)]
    got = bat.encode_pinned_batch([x.pin_memory(), y.pin_memory(), x])
    assert [g.numpy().tobytes() for g in got] == want
    back = bat.decode_pinned_batch(got)
    assert [t.view(torch.int16).numpy().tobytes() for t in back] == [seq.decode(w) for w in want]
    # non-blocking calls, a decode queued between an encode and its result
    asy = DitheredNBitCodec(hidden_dim=hidden, bits=bits)
    first = asy.encode_pinned_batch([x.pin_memory(), y.pin_memory()])
    pend_dec = asy.decode_pinned_batch(first, wait=False)
    pend_enc = asy.encode_pinned_batch([x], wait=False)
    assert [t.view(torch.int16).numpy().tobytes() for t in pend_dec.result()] == [seq.decode(w) for w in want[:2]]
    assert pend_enc.result()[0].numpy().tobytes() == want[2]
    # blobs handed from an encode to a decode on another stream without a host wait
    # (the decode's reads ordered after the encode's copies on the GPU), over a
    # three-deep rotation of blob buffers as a streaming caller uses them
    nw = DitheredNBitCodec(hidden_dim=hidden, bits=bits)
    bufs = [[torch.empty(len(w) + 64, dtype=torch.uint8, pin_memory=True) for w in want[:2]] for _ in range(3)]
    outs = [[torch.empty(t.numel(), dtype=torch.bfloat16, pin_memory=True) for t in (x, y)] for _ in range(2)]
    side = torch.cuda.Stream(cuda)
    ref = DitheredNBitCodec(hidden_dim=hidden, bits=bits)  # same call sequence, same seeds
    wants = [ref.encode(bits_of(t).tobytes()) for _ in range(3) for t in (x, y)]
    blobs = nw.encode_pinned_batch([x.pin_memory(), y.pin_memory()], bufs[0], host_sync=False)
    got_blobs, pend = [], []
    for s_ in range(1, 4):
        pe = nw.encode_pinned_batch([x.pin_memory(), y.pin_memory()], bufs[s_ % 3], wait=False, host_sync=False) \
            if s_ < 3 else None
        with torch.cuda.stream(side):
            pend.append((blobs, nw.decode_pinned_batch(blobs, outs[s_ % 2], wait=False)))
        if pe is not None:
            blobs = pe.result()
        prev_blobs, pd = pend.pop(0)
        decoded = [t.view(torch.int16).numpy().tobytes() for t in pd.result()]
        got_blobs.append([bb.numpy().tobytes() for bb in prev_blobs])
        assert decoded == [seq.decode(w) for w in got_blobs[-1]]
    assert [b_ for pair in got_blobs for b_ in pair] == wants
    from ashkv.codecs.nbit_dithered import sync_host_blobs
    last = nw.encode_pinned_batch([x.pin_memory()], [bufs[0][0]], host_sync=False)
    sync_host_blobs(last)
    assert last[0].numpy().tobytes() == ref.encode(bits_of(x).tobytes())
    c = DitheredINT2Codec()
    u = torch.rand(x.numel() // 128 * 128)
    assert c.encode_pinned(x, uniform=u).numpy().tobytes() == c.encode(data, uniform=u)
    assert DitheredNBitCodec().encode_pinned(torch.empty(0, dtype=torch.bfloat16)).numpy().tobytes() == bytes(8)


def test_nbit_pinned_streaming_loop_keeps_buffers_alive(cuda):
    """A decode queued with wait=False and then an encode queued with wait=False,
    repeated: the decode's device status word (read back on a side stream after the
    call returns) and every other side-stream buffer stay reserved until their
    copies finish, so the encode's allocations cannot land on them (a use-after-free
    here showed up as spurious index-range/overflow flags)."""
    n = 1 << 22
    x = rand_bf16(n, 81, "outliers").pin_memory()
    y = rand_bf16(n, 82, "wide").pin_memory()
    ref = DitheredNBitCodec(hidden_dim=128, bits=4)
    want = [[ref.encode(bits_of(t).tobytes()) for t in (x, y)] for _ in range(7)]
    c = DitheredNBitCodec(hidden_dim=128, bits=4)
    bufs = [[torch.empty(len(w) + 64, dtype=torch.uint8, pin_memory=True) for w in want[0]] for _ in range(2)]
    outs = [torch.empty(n, dtype=torch.bfloat16, pin_memory=True) for _ in range(2)]
    blobs = c.encode_pinned_batch([x, y], bufs[0])
    for s_ in range(1, 7):
        pd = c.decode_pinned_batch(blobs, outs, wait=False)
        pe = c.encode_pinned_batch([x, y], bufs[s_ % 2], wait=False)
        got = [t.view(torch.int16).numpy().tobytes() for t in pd.result()]
        assert got == [ref.decode(w) for w in want[s_ - 1]]
        blobs = pe.result()
        assert [b.numpy().tobytes() for b in blobs] == want[s_]


def test_nbit_config3_full_size_int2_properties(cuda):
    """INT2 workload at full size: 80 layers x K,V x [2048 pages, 16, 8 heads, 128],
    N(0, s^2) with s ~ U[0.5, 2] per (layer, K/V, head), 5.37 G elements in 160
    tensors, each encoded with the INT2 codec's dither seed and decoded back.
    Per tensor: outliers restored bit-exactly, every other element within one
    quantisation step of its group; a sample of buckets bit-exact against the oracle."""
    pages, T, H, D = 2048, 16, 8, 128
    n = pages * T * H * D
    g = torch.Generator(device=cuda).manual_seed(0)
    sd_gen = torch.Generator().manual_seed(1)
    total_out = 0
    for layer in range(80):
        for kv in range(2):
            sd = torch.empty(H).uniform_(0.5, 2.0, generator=sd_gen).to(cuda)
            x = (torch.randn(pages, T, H, D, generator=g, device=cuda) * sd.view(1, 1, H, 1)).to(torch.bfloat16)
            x = x.view(-1)
            enc = nb.encode_groups(x, 2, 3.0, seed=42)
            dec = nb.decode_groups(enc)
            idx, val, total = nb.flatten_outliers(enc)
            t = int(total.item())
            total_out += t
            ii = idx[:t].long()
            assert torch.equal(dec[ii].view(torch.int16), x[ii].view(torch.int16))
            delta = enc.scales.float().repeat_interleave(32)
            err = (dec.float() - x.float()).abs()
            err[ii] = 0.0
            assert bool((err <= delta * 1.01).all()), (layer, kv)
            assert int(enc.status.item()) == 0
            if layer % 27 == 0:
                xs, sc, codes = bits_of(x), bits_of(enc.scales), enc.codes.cpu().numpy()
                for lo in range(0, n, n // 4):
                    u = oracle.philox_dither(8192, 42, lo)
                    osc, ocodes, _, _ = oracle.nbit_encode(xs[lo:lo + 8192], 2, u, 3.0)
                    assert np.array_equal(sc[lo // 32:(lo + 8192) // 32], osc)
                    assert np.array_equal(codes[lo // 4:(lo + 8192) // 4], ocodes)
            del x, enc, dec, err, delta
    # 3-sigma tails of Gaussian groups: a fraction of a percent of the elements
    assert 0 < total_out < 80 * 2 * n // 100


def test_nbit_codec_seeding_policy(cuda):
    x = bits_of(rand_bf16(4 * 128, 51)).tobytes()
    c = DitheredNBitCodec()
    a, b = c.encode(x), c.encode(x)
    assert a != b  # seed 42 + call count: the dither differs between calls
    c2 = DitheredINT2Codec()
    assert c2.encode(x) == c2.encode(x)  # fixed seed 42
    assert DitheredNBitCodec().encode(b"") == b"\x00" * 8


@pytest.mark.parametrize("offset_words,n_words", [(0, 1), (1, 7), (3, 9), (7, 8), (5, 1000), (0, 1 << 20), (2, (1 << 20) + 3)])
def test_fill32_head_body_tail(cuda, offset_words, n_words):
    """Every word of [offset, offset + n) gets the pattern; the words around it do not."""
    buf = torch.zeros(offset_words + n_words + 16, dtype=torch.int32, device=cuda)
    view = buf[offset_words:offset_words + n_words]
    _native.fill32(view, 0xA5A5_5A5A)
    got = buf.cpu().numpy().view(np.uint32)
    assert (got[offset_words:offset_words + n_words] == 0xA5A55A5A).all()
    assert (got[:offset_words] == 0).all() and (got[offset_words + n_words:] == 0).all()


def _bits_equal_or_both_nan(a: np.ndarray, b: np.ndarray) -> bool:
    """bf16 bit arrays equal, NaN against NaN whatever the payload (CUDA writes 0x7FFF)."""
    nan_a = (a & 0x7F80) == 0x7F80
    nan_a &= (a & 0x007F) != 0
    nan_b = ((b & 0x7F80) == 0x7F80) & ((b & 0x007F) != 0)
    return bool(np.all((a == b) | (nan_a & nan_b)))


@pytest.mark.parametrize("bits", [2, 4, 8])
@pytest.mark.parametrize("mode", ["tensor", "philox"])
def test_nbit_nan_inf_groups_match_oracle(cuda, bits, mode):
    """Groups holding NaN (quiet, signalling pattern, negative with payload), +-inf, both,
    or only NaN, among ordinary groups: codes and outlier lists exact, scales equal or
    both NaN."""
    n_groups = 64 * 32
    x = rand_bf16(n_groups * 32, 41 + bits, "outliers")
    b = bits_of(x).reshape(n_groups, 32).copy()
    b[1, 0] = 0x7FC0               # quiet NaN
    b[3, 31] = 0xFFC1              # negative NaN with a payload
    b[5, 7] = 0x7FA0               # signalling-NaN pattern
    b[7, 3] = 0x7F80               # +inf
    b[9, 12] = 0xFF80              # -inf
    b[11, 2], b[11, 9] = 0x7F80, 0xFF80
    b[13, 4], b[13, 5] = 0x7FC0, 0x7F80
    b[15, :] = 0x7FC0              # every element NaN
    b[17, :] = 0x7F80              # every element +inf
    b[100::97, 6] = 0x7FC0         # NaN sprinkled over later buckets
    b = b.reshape(-1)
    xt = torch.from_numpy(b.view(np.int16).copy()).view(torch.bfloat16).to(cuda)
    if mode == "tensor":
        u = torch.rand(b.size, generator=torch.Generator().manual_seed(bits))
        enc = nb.encode_groups(xt, bits, 3.0, uniform=u.to(cuda))
        un = u.numpy()
    else:
        enc = nb.encode_groups(xt, bits, 3.0, seed=99, dither_offset=0)
        un = oracle.philox_dither(b.size, 99, 0)
    osc, ocodes, oidx, ovals = oracle.nbit_encode(b, bits, un, 3.0)
    assert _bits_equal_or_both_nan(bits_of(enc.scales), osc)
    assert np.array_equal(enc.codes[: ocodes.size].cpu().numpy(), ocodes)
    idx, val, total = nb.flatten_outliers(enc)
    t = int(total.item())
    assert t == oidx.size and np.array_equal(idx[:t].cpu().numpy(), oidx)
    assert np.array_equal(val[:t].cpu().numpy().view(np.uint16), ovals)
