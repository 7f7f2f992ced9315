"""The CPU oracle against golden vectors produced by the reference itself.

tests/golden/make_golden.py ran the reference's own codec/policy/checksum
code (N-bit and INT2 codecs on the CPU with an injected dither; the Triton
INT8 kernel under Triton's interpreter) and stored inputs and outputs.
These tests pin the oracle that the GPU parity tests compare against.
"""
from __future__ import annotations

import numpy as np
import pytest

import oracle
from conftest import GOLDEN

NBIT = np.load(GOLDEN / "nbit.npz")
INT8 = np.load(GOLDEN / "int8.npz")
POLICY = np.load(GOLDEN / "policy.npz")
XXH = np.load(GOLDEN / "xxh64.npz")
F84 = np.load(GOLDEN / "fp8_int4.npz")


@pytest.mark.parametrize("ci", range(int(NBIT["nbit_n_cases"])))
def test_nbit_oracle_matches_reference_blob(ci):
    pre = f"nbit_{ci}_"
    bits, hidden, _is_int2, n, _trail = (int(v) for v in NBIT[pre + "meta"])
    sigma = float(NBIT[pre + "sigma"])
    blob = NBIT[pre + "blob"].tobytes()
    x = NBIT[pre + "src"][:n]
    sc, codes, idx, vals = oracle.nbit_encode(x, bits, NBIT[pre + "u"], sigma)
    num_tokens = n // hidden
    assert oracle.nbit_blob(num_tokens, sc, codes, idx, vals) == blob  # every byte, incl. outlier list
    dec = oracle.nbit_decode(sc, codes, bits, idx, vals)
    assert dec.tobytes() == NBIT[pre + "decoded"].tobytes()


def test_nbit_golden_covers_outliers_and_all_widths():
    widths, outliers = set(), 0
    for ci in range(int(NBIT["nbit_n_cases"])):
        pre = f"nbit_{ci}_"
        widths.add(int(NBIT[pre + "meta"][0]))
        outliers += oracle.nbit_parse_blob(NBIT[pre + "blob"].tobytes(), int(NBIT[pre + "meta"][1]))[2].size
    assert widths == {2, 4, 8} and outliers > 1000


@pytest.mark.parametrize("ci", range(int(INT8["int8_n_cases"])))
def test_int8_oracle_matches_reference_kernel(ci):
    pre = f"int8_{ci}_"
    rows, L, _ = (int(v) for v in INT8[pre + "meta"])
    src = INT8[pre + "src"].reshape(rows, L)
    codes, scales = oracle.int8_encode(src, L, src_fp16=True, scale_fp16=True)
    assert np.array_equal(scales, INT8[pre + "scales"])
    # Where v*127 overflows fp16 (|v| > 65504/127) the product is inf; the
    # interpreter's numpy cast of that yields 0, while Triton on the GPU (and the
    # oracle, pinned to it by int8_bf16.npz) converts to int32 and keeps the low
    # byte: +inf -> -1, -inf -> 0.  Everywhere else the codes must be identical.
    x = src.view(np.float16).astype(np.float32)
    overflow = np.abs(x) * 127.0 > 65504.0
    assert np.array_equal(codes[~overflow], INT8[pre + "codes"][~overflow])
    assert np.array_equal(codes[overflow], np.where(x[overflow] > 0, -1, 0).astype(np.int8))


def test_int8_decode_formula():
    rng = np.random.default_rng(0)
    codes = rng.integers(-128, 128, size=(16, 128)).astype(np.int8)
    scales = (rng.random(16).astype(np.float32) * 4).astype(np.float32)
    sbits = np.array([oracle.lib().oracle_f32_to_bf16(float(s)) for s in scales], dtype=np.uint16)
    out = oracle.int8_decode(codes, sbits)
    s32 = (sbits.astype(np.uint32) << 16).view(np.float32)
    want = (codes.astype(np.float32) * s32[:, None]) / np.float32(127.0)
    got = (out.astype(np.uint32) << 16).view(np.float32)
    assert np.all(np.abs(got - want) <= np.abs(want) * 2.0 ** -8)


def test_int8_oracle_row_maximum_skips_every_nan():
    """The row maximum ignores quiet and signalling NaNs alike (the GPU max
    instruction's rule, which Triton's tl.maximum lowers to), NaN codes are 0,
    and an all-NaN row falls to the 1e-8 floor."""
    L = 128
    rng = np.random.default_rng(3)
    x = rng.standard_normal((4, L)).astype(np.float32)
    bits = (x.view(np.uint32) >> 16).astype(np.uint16)  # truncated to bf16 bits
    bits[0, ::2] = 0x7FA0           # signalling-NaN pattern on every other element
    bits[1, 5] = 0xFFC1             # negative quiet NaN with a payload
    bits[2, :] = 0x7FC0             # every element NaN
    codes, scales = oracle.int8_encode(bits, L)
    vals = (bits.astype(np.uint32) << 16).view(np.float32)
    for r in (0, 1):
        finite = vals[r][~np.isnan(vals[r])]
        want = oracle.lib().oracle_f32_to_bf16(float(np.abs(finite).max()))
        assert scales[r] == want
        assert np.all(codes[r][np.isnan(vals[r])] == 0)
    assert scales[2] == oracle.lib().oracle_f32_to_bf16(1e-8)
    assert np.all(codes[2] == 0)


def test_policy_oracle_matches_reference():
    z = POLICY
    R = oracle.score(z["policy_T"], z["policy_S"], z["policy_N"], z["policy_P"], 0.7, 0.1, 0.1, 0.1)
    assert np.array_equal(R, z["policy_R"], equal_nan=True)
    nc, nh = oracle.controller_tables([tuple(k) for k in z["policy_codec_keys"]])
    assert np.array_equal(nc, z["policy_next_colder"]) and np.array_equal(nh, z["policy_next_hotter"])
    for i, p in enumerate(z["policy_pressures"]):
        t = oracle.desired_tiers(R, z["policy_cur"], float(p), 0.72, 0.33, 0.04, 0.95, nc, nh)
        assert np.array_equal(t, z[f"policy_target_{i}"]), p
    R2 = oracle.score(z["policy_T"], z["policy_S"], z["policy_N"], z["policy_P"], 0.55, 0.15, 0.2, 0.1)
    assert np.array_equal(R2, z["policy_R2"], equal_nan=True)
    t2 = oracle.desired_tiers(R2, z["policy_cur"], 0.963, 0.61, 0.29, 0.03, 0.9, nc, nh)
    assert np.array_equal(t2, z["policy_target_alt"])


def test_xxh64_oracle_matches_reference_checksum():
    off = 0
    for L, digest in zip(XXH["xxh64_lengths"], XXH["xxh64_digest"]):
        L = int(L)
        assert oracle.xxh64(XXH["xxh64_data"][off:off + L].tobytes()) == int(digest), L
        off += L


def test_xxh64_known_answers():
    # Published XXH64 test values (seed 0).
    assert oracle.xxh64(b"") == 0xEF46DB3751D8E999
    assert oracle.xxh64(b"abc") == 0x44BC2CF5AD770999


def test_philox_known_answers():
    # Random123 known-answer vectors for philox4x32-10.
    assert list(oracle.philox4x32_10([0, 0, 0, 0], [0, 0])) == [0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8]
    assert list(oracle.philox4x32_10([0xFFFFFFFF] * 4, [0xFFFFFFFF] * 2)) == [
        0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD]
    assert list(oracle.philox4x32_10([0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344],
                                     [0xA4093822, 0x299F31D0])) == [0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1]


def test_philox_dither_range_and_offset():
    u = oracle.philox_dither(4096, seed=7)
    assert u.min() > 0.0 and u.max() < 1.0
    assert np.array_equal(oracle.philox_dither(64, seed=7, offset=1024), u[1024:1088])
    assert abs(float(u.mean()) - 0.5) < 0.02
    # centred 8-bit uniforms: U = (b + 0.5) / 256, b = byte e & 15 of Philox4x32-10(counter e >> 4)
    b = u * 256.0 - 0.5
    assert np.array_equal(b, np.round(b)) and b.min() >= 0 and b.max() <= 255
    words = oracle.philox4x32_10([3, 0, 0, 0], [7, 0])
    assert np.array_equal(b[48:64].astype(np.uint8), words.view(np.uint8))


def test_outlier_bound_holds_on_adversarial_groups():
    rng = np.random.default_rng(5)
    worst = 0
    for _ in range(200):
        x = rng.standard_normal((256, 32)).astype(np.float32)
        k = rng.integers(1, 6)
        x[:, :k] *= 1e3
        xb = ((x.view(np.uint32) + 0x7FFF + ((x.view(np.uint32) >> 16) & 1)) >> 16).astype(np.uint16)
        _, _, idx, _ = oracle.nbit_encode(xb, 4, np.full(xb.size, 0.5, np.float32), 3.0)
        if idx.size:
            worst = max(worst, np.bincount(idx // 32).max())
    assert worst <= oracle.max_outliers_per_group(3.0)


def test_fp8_oracle_matches_reference_on_every_bf16_pattern():
    allb = np.arange(65536, dtype=np.uint16)
    np.testing.assert_array_equal(oracle.fp8_encode(allb), F84["fp8_encode_all"])


def test_fp8_decode_oracle_matches_reference_on_every_code():
    dec = oracle.fp8_decode(np.arange(256, dtype=np.uint8))
    ref = F84["fp8_decode_all"]
    nan = np.array([0x7F, 0xFF])
    finite = np.setdiff1d(np.arange(256), nan)
    np.testing.assert_array_equal(dec[finite], ref[finite])
    # The fixture comes from torch's CPU cast (NaN -> 0x7FC0); the reference runs
    # the cast on CUDA when a GPU is present, which writes 0x7FFF.
    assert set(ref[nan].tolist()) == {0x7FC0}
    assert set(dec[nan].tolist()) == {oracle.FP8_NAN_BF16_CUDA}
    assert set(oracle.fp8_decode(nan.astype(np.uint8), nan_bits=0x7FC0).tolist()) == {0x7FC0}


@pytest.mark.parametrize("ci", range(len(F84["int4_group_size"])))
def test_int4_oracle_matches_reference_blob(ci):
    gs = int(F84["int4_group_size"][ci])
    x = F84[f"int4_in_{ci}"]
    scales, packed, total = oracle.int4_encode(x, gs)
    blob = oracle.int4_blob(scales, packed, total)
    assert blob == F84[f"int4_blob_{ci}"].tobytes()
    np.testing.assert_array_equal(oracle.int4_decode(scales, packed, gs), F84[f"int4_dec_{ci}"])


def test_int4_oracle_decodes_random_reference_blobs():
    blob = F84["int4_rand_blob"].tobytes()
    n_groups, n_values = np.frombuffer(blob[:8], np.uint32)
    sc = np.frombuffer(blob[8:8 + 2 * n_groups], np.uint16)
    packed = np.frombuffer(blob[8 + 2 * n_groups:], np.uint8)
    np.testing.assert_array_equal(oracle.int4_decode(sc, packed, int(n_values // n_groups)), F84["int4_rand_dec"])


def test_int4_golden_covers_special_values():
    specials = [ci for ci in range(len(F84["int4_group_size"]))
                if np.any((F84[f"int4_in_{ci}"] & 0x7F80) == 0x7F80)]
    assert specials, "no NaN/inf case in the INT4 fixture"
    assert F84["int4_empty_blob"].tobytes() == b"\0\0\0\0"


def test_feature_oracle_properties():
    """The saliency oracle conserves probability mass (every visible query row sums
    to 1) and matches a float64 evaluation; novelty is 0 for repeated keys."""
    import torch
    g = torch.Generator().manual_seed(0)
    q = torch.randn(40, 4, 16, generator=g)
    k = torch.randn(50, 2, 16, generator=g)
    s = oracle.attention_saliency(q, k)
    assert abs(float(s.sum()) - 4 * 40) < 1e-3
    # float64 restatement
    qh = q.double().transpose(0, 1)
    kh = k.double().transpose(0, 1).repeat_interleave(2, dim=0)
    sc = qh @ kh.transpose(-2, -1) / 4.0
    mask = torch.arange(50).view(1, -1) > (torch.arange(40).view(-1, 1) + 10)
    p = torch.softmax(sc.masked_fill(mask, float("-inf")), dim=-1).sum(dim=(0, 1))
    assert np.allclose(s.numpy(), p.numpy(), rtol=1e-5, atol=1e-6)
    kk = torch.ones(32, 2, 16)
    S, N = oracle.page_features(kk, 16, np.arange(32, dtype=np.float64))
    assert np.all(N == 0) and S.max() == 1.0


# ---------------------------------------------------------------- B200 fixtures
# Produced by tests/golden/make_golden_gpu.py: the reference's Triton INT8
# kernels, SGLang hooks, simulator and N-bit codecs executed on a B200.
INT8_GPU = np.load(GOLDEN / "int8_bf16.npz")
HOOKS_GPU = np.load(GOLDEN / "hooks_int8.npz")
SAL_GPU = np.load(GOLDEN / "saliency.npz")
NBIT_CUDA = np.load(GOLDEN / "nbit_cuda.npz")


def test_b200_fixture_every_triton_config_agrees():
    assert INT8_GPU["config_mismatches"].size == 0
    assert "B200" in str(INT8_GPU["meta_gpu"])


@pytest.mark.parametrize("L", [int(v) for v in INT8_GPU["row_lens"]])
@pytest.mark.parametrize("sname", ["bf16", "fp16"])
def test_int8_oracle_matches_b200_reference_kernel(L, sname):
    """bf16 rows (normal, NaN, +-inf, subnormal, zero, overflowing products, near-.5
    quotients, absmax under the floor): scales identical, codes identical except one
    apart at tie-zone elements (the reference divides with div.full.f32)."""
    x = INT8_GPU[f"enc_in_L{L}"]
    codes, scales, tie = oracle.int8_encode(x, L, scale_fp16=sname == "fp16", with_ties=True)
    assert np.array_equal(scales, INT8_GPU[f"enc_scales_L{L}_{sname}"])
    ok, n_diff = oracle.int8_codes_agree(INT8_GPU[f"enc_codes_L{L}_{sname}"], codes, tie)
    assert ok and n_diff <= 8, n_diff
    assert tie.sum() > 0  # the fixture does exercise the tie zone


@pytest.mark.parametrize("sname", ["bf16", "fp16"])
def test_int8_oracle_decode_matches_b200_reference_kernel(sname):
    sc = INT8_GPU[f"dec_scales_{sname}"]
    codes = np.tile(INT8_GPU["dec_codes_row"], (sc.size, 1))
    got = oracle.int8_decode(codes, sc, scale_fp16=sname == "fp16")
    assert np.array_equal(got, INT8_GPU[f"dec_out_{sname}"])


def hook_case(i: int):
    z = HOOKS_GPU
    layers, cap, hcap, H, D, n = (int(v) for v in z[f"case{i}_shape"])
    return z, layers, H, D, n


@pytest.mark.parametrize("i", range(int(HOOKS_GPU["n_cases"])))
def test_hook_slot_oracle_matches_b200_reference_hooks(i):
    """Host slot bytes of the reference's demote_hook: [fp16 scales at the flat
    positions | int8 codes | zeros]; the scale entries past the last token are
    uninitialised in the reference (torch.empty) and are not compared."""
    z, layers, H, D, n = hook_case(i)
    for kv in ("k", "v"):
        dev, idx = z[f"case{i}_dev_{kv}"], z[f"case{i}_dev_idx"]
        slots = z[f"case{i}_host_{kv}"].reshape(n, layers, H * D).view(np.uint8).reshape(n, layers, 2 * H * D)
        defined = np.repeat(np.arange(n * H).reshape(n, H) < n, 2, axis=1)
        for l in range(layers):
            rows = dev[l][idx].reshape(n, H * D)
            codes, scales, tie = oracle.int8_encode(rows, H * D, scale_fp16=True, with_ties=True)
            flat = np.zeros(n * H, np.uint16)
            flat[:n] = scales
            want_sc = flat.reshape(n, H).view(np.uint8).reshape(n, 2 * H)
            got = slots[:, l]
            assert np.array_equal(got[:, :2 * H][defined], want_sc[defined])
            ok, _ = oracle.int8_codes_agree(got[:, 2 * H:2 * H + H * D].copy(), codes, tie)
            assert ok, (kv, l)
            assert not got[:, 2 * H + H * D:].any()
            # promote_hook restores the decode of exactly these stored bytes
            dec = oracle.int8_decode(got[:, 2 * H:2 * H + H * D].copy().view(np.int8),
                                     got[:, :2 * H].copy().view(np.uint16).reshape(-1)[:n], scale_fp16=True)
            assert np.array_equal(dec, z[f"case{i}_prom_{kv}"][l].reshape(n, H * D))


@pytest.mark.parametrize("i", range(int(SAL_GPU["n_cases"])))
def test_saliency_oracle_matches_b200_reference_simulator(i):
    """The simulator's per-key attention mass (fp32 matmul + softmax on CUDA)."""
    import torch
    S, H, D = (int(v) for v in SAL_GPU[f"case{i}_shape"])
    q = torch.from_numpy(SAL_GPU[f"case{i}_q"].view(np.int16)).view(torch.bfloat16).view(S, H, D)
    k = torch.from_numpy(SAL_GPU[f"case{i}_k"].view(np.int16)).view(torch.bfloat16).view(S, H, D)
    ref = SAL_GPU[f"case{i}_saliency"]
    fin = np.isfinite(ref)
    assert fin.sum() == S - 33  # the simulator pins key 0 and the last 32 keys to +inf
    got = oracle.attention_saliency(q, k).numpy()
    assert np.abs(got[fin] - ref[fin]).max() <= 1e-5 * ref[fin].max()


@pytest.mark.parametrize("name,bits", [("nbit4", 4), ("int2", 2)])
def test_nbit_oracle_matches_reference_run_on_cuda(name, bits):
    """DitheredNBitCodec(bits=4) / DitheredINT2Codec run natively on CUDA with their
    own generator: given the uniforms they drew, the oracle's blob is identical."""
    x = NBIT_CUDA["input"]
    U = NBIT_CUDA[f"{name}_uniform"]
    blob = NBIT_CUDA[f"{name}_blob"].tobytes()
    sc, codes, idx, vals = oracle.nbit_encode(x, bits, U, 3.0)
    assert oracle.nbit_blob(x.size // 128, sc, codes, idx, vals) == blob
    assert np.array_equal(oracle.nbit_decode(sc, codes, bits, idx, vals), NBIT_CUDA[f"{name}_decoded"])
