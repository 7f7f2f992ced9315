"""GPU parity against the reference's own outputs on a B200, exactly.

The fixtures were produced by ``tests/golden/make_golden_gpu.py`` running the
reference package itself on a B200: its Triton INT8 kernels (autotuned path;
the script checked that all nine autotune configurations agree), its SGLang
``demote_hook`` / ``promote_hook`` on mock pools, its simulator's attention
mass, and its N-bit / INT2 codecs run natively on CUDA with the uniforms they
drew recorded.  Here the sm_100a kernels, through the C ABI, must reproduce
them: INT8 codes and scales bit for bit (ties included: the kernels divide as
the reference's Triton code does on the GPU), host slot bytes and promoted
rows bit for bit, N-bit blobs and decoded bytes bit for bit, and the
tensor-core saliency within 1e-4 of the largest value.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import GOLDEN

from ashkv import _native
from ashkv.adapters.sglang.hooks import SGLangHooks
from ashkv.codecs import DitheredINT2Codec, DitheredNBitCodec
from ashkv.codecs import int8 as int8_mod
from ashkv.runtime import features

pytestmark = pytest.mark.gpu

INT8_GPU = np.load(GOLDEN / "int8_bf16.npz")
HOOKS_GPU = np.load(GOLDEN / "hooks_int8.npz")
SAL_GPU = np.load(GOLDEN / "saliency.npz")
NBIT_CUDA = np.load(GOLDEN / "nbit_cuda.npz")


def u16(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def bf16_dev(bits: np.ndarray, dev) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(bits, np.uint16).view(np.int16)).view(torch.bfloat16).to(dev)


@pytest.mark.parametrize("L", [int(v) for v in INT8_GPU["row_lens"]])
@pytest.mark.parametrize("sname", ["bf16", "fp16"])
def test_int8_encode_equals_reference_triton_on_b200(cuda, L, sname):
    x = INT8_GPU[f"enc_in_L{L}"]
    n = x.shape[0]
    sdt = torch.bfloat16 if sname == "bf16" else torch.float16
    codes, scales = int8_mod.encode_rows(bf16_dev(x, cuda).view(n, L), scale_dtype=sdt)
    assert np.array_equal(codes.cpu().numpy(), INT8_GPU[f"enc_codes_L{L}_{sname}"])
    assert np.array_equal(u16(scales), INT8_GPU[f"enc_scales_L{L}_{sname}"])
    # the launcher seam with the Triton kernels' call shape gives the same bytes
    enc, _ = int8_mod._get_kernels()
    c2 = torch.empty((n, L), dtype=torch.int8, device=cuda)
    s2 = torch.empty((n,), dtype=sdt, device=cuda)
    enc[(n,)](bf16_dev(x, cuda).view(n, L), c2, s2, n, L)
    assert torch.equal(c2, codes) and torch.equal(s2.view(torch.int16), scales.view(torch.int16))


@pytest.mark.parametrize("sname", ["bf16", "fp16"])
def test_int8_decode_equals_reference_triton_on_b200(cuda, sname):
    sc = INT8_GPU[f"dec_scales_{sname}"]
    sdt = torch.bfloat16 if sname == "bf16" else torch.float16
    codes = torch.from_numpy(np.tile(INT8_GPU["dec_codes_row"], (sc.size, 1))).to(cuda)
    out = int8_mod.decode_rows(codes, torch.from_numpy(sc.view(np.int16)).view(sdt).to(cuda))
    assert np.array_equal(u16(out), INT8_GPU[f"dec_out_{sname}"])


class _DevPool:
    def __init__(self, k, v, H, D, dev):
        self.head_num, self.head_dim, self.layer_num = H, D, k.shape[0]
        self.k_buffer = [bf16_dev(k[l], dev).view(-1, H, D) for l in range(k.shape[0])]
        self.v_buffer = [bf16_dev(v[l], dev).view(-1, H, D) for l in range(v.shape[0])]


class _HostPool:
    def __init__(self, layers, cap, H, D):
        self.k_buffer = torch.zeros((cap, layers, H, D), dtype=torch.bfloat16)
        self.v_buffer = torch.zeros((cap, layers, H, D), dtype=torch.bfloat16)


@pytest.mark.parametrize("i", range(int(HOOKS_GPU["n_cases"])))
@pytest.mark.parametrize("compact", [False, True])
def test_hooks_equal_reference_hooks_on_b200(cuda, tmp_path, monkeypatch, i, compact):
    """demote_hook writes the reference's host slot bytes (its uninitialised scale
    entries past the last token excluded); promote_hook restores its rows."""
    monkeypatch.chdir(tmp_path)
    z = HOOKS_GPU
    layers, cap, hcap, H, D, n = (int(v) for v in z[f"case{i}_shape"])
    dp = _DevPool(z[f"case{i}_dev_k"], z[f"case{i}_dev_v"], H, D, cuda)
    hp = _HostPool(layers, hcap, H, D)
    d_idx = torch.from_numpy(z[f"case{i}_dev_idx"]).to(cuda)
    h_idx = torch.from_numpy(z[f"case{i}_host_idx"])
    hooks = SGLangHooks()
    hooks.compact_host_slots = compact
    assert hooks.demote_hook(dp, hp, h_idx, d_idx, "MHA")
    defined = np.ones((n, 2 * H * D), bool)
    defined[:, :2 * H] = np.repeat(np.arange(n * H).reshape(n, H) < n, 2, axis=1)
    for kv in ("k", "v"):
        got = u16(getattr(hp, f"{kv}_buffer")[h_idx]).reshape(n, layers, H * D).view(np.uint8)
        want = z[f"case{i}_host_{kv}"].reshape(n, layers, H * D).view(np.uint8)
        for l in range(layers):
            assert np.array_equal(got[:, l][defined], want[:, l][defined]), (kv, l)
    for t in dp.k_buffer + dp.v_buffer:
        t.zero_()
    for l in range(layers):
        assert hooks.promote_hook(dp, hp, h_idx, d_idx, l, "MHA")
    for kv in ("k", "v"):
        for l in range(layers):
            got = u16(getattr(dp, f"{kv}_buffer")[l][d_idx])
            assert np.array_equal(got, z[f"case{i}_prom_{kv}"][l]), (kv, l)


@pytest.mark.parametrize("i", range(int(SAL_GPU["n_cases"])))
def test_saliency_kernel_matches_reference_simulator_on_b200(cuda, i):
    S, H, D = (int(v) for v in SAL_GPU[f"case{i}_shape"])
    q = bf16_dev(SAL_GPU[f"case{i}_q"], cuda).view(S, H, D)
    k = bf16_dev(SAL_GPU[f"case{i}_k"], cuda).view(S, H, D)
    got = features.attention_saliency(q, k).cpu().numpy()
    ref = SAL_GPU[f"case{i}_saliency"]
    fin = np.isfinite(ref)
    assert np.abs(got[fin] - ref[fin]).max() <= 1e-4 * ref[fin].max()


@pytest.mark.parametrize("name,bits", [("nbit4", 4), ("int2", 2)])
def test_nbit_blob_equals_reference_run_on_cuda(cuda, name, bits):
    """Given the uniforms the reference's CUDA generator drew, the bytes API returns
    the reference's blob byte for byte and decodes it to the reference's bytes."""
    codec = DitheredNBitCodec(bits=4) if bits == 4 else DitheredINT2Codec()
    x = NBIT_CUDA["input"]
    U = torch.from_numpy(NBIT_CUDA[f"{name}_uniform"].astype(np.float32))
    blob = codec.encode(x.tobytes(), uniform=U)
    assert blob == NBIT_CUDA[f"{name}_blob"].tobytes()
    assert np.array_equal(np.frombuffer(codec.decode(blob), np.uint16), NBIT_CUDA[f"{name}_decoded"])
