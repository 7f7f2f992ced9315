"""Generate the golden fixtures in tests/golden/ by running the reference ASH-KV code.

Run in a container that has the reference source tree (read-only is fine):

    python tests/golden/make_golden.py --reference <reference tree>

(or set ASHKV_REFERENCE to that tree instead of passing --reference)

The reference is imported as the ``ashkv`` package from that tree, so this
script must not import this repository's own ``ashkv``.  It produces:

* ``nbit.npz``   — DitheredNBitCodec (2/4/8 bits, several sigma/hidden_dim)
  and DitheredINT2Codec encode+decode.  The reference codec body runs
  unchanged on the CPU: ``Tensor.cuda`` becomes the identity, CUDA
  ``torch.empty`` is redirected to the CPU, and ``torch.rand`` returns an
  injected ``U`` so that ``noise = (U - 0.5) * delta`` is known exactly.
* ``int8.npz``   — the reference Triton ``_int8_encode_kernel`` executed by
  Triton's interpreter (``TRITON_INTERPRET=1``) on fp16 rows with fp16 scale
  buffers (the SGLang hooks' scale type).  The interpreter mishandles bf16
  (it truncates instead of rounding), so no bf16 case is generated here.
* ``policy.npz`` — ``score_vectorized`` and ``desired_tiers`` over seeded
  page features at several pressures, with the controller lookup tables
  compiled by ``compile_controller``.
* ``xxh64.npz``  — ``ashkv.codecs.checksum.checksum`` (xxhash 3.x XXH64,
  seed 0) over seeded byte strings of many lengths.
* ``fp8_int4.npz`` — ``FP8Codec`` over all 65,536 bf16 bit patterns and all
  256 codes (torch's CPU casts; the same conversion function torch runs on
  CUDA, except that CUDA writes a NaN bf16 as 0x7FFF), and ``INT4Codec``
  encode/decode blobs for seeded inputs, group sizes 7..128, special values,
  and decode of random blobs.

Inputs are seeded synthetic data; the script is deterministic.
"""
from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def _bf16_bits(t) -> np.ndarray:
    import torch
    return t.to(torch.bfloat16).contiguous().view(torch.int16).numpy().view(np.uint16).copy()


class _CpuShim:
    """Run the reference codec bodies on the CPU with an injected uniform tensor."""

    def __init__(self):
        import torch
        self.torch = torch
        self.U = None

    def __enter__(self):
        torch = self.torch
        self._cuda = torch.Tensor.cuda
        self._rand = torch.rand
        self._empty = torch.empty
        shim = self

        def cuda(self_t, *a, **k):
            return self_t

        def rand(*size, generator=None, device=None, dtype=None, **kw):
            if len(size) == 1 and isinstance(size[0], (tuple, list, torch.Size)):
                size = tuple(size[0])
            u = shim.U
            assert u is not None and tuple(u.shape) == tuple(size), (u.shape if u is not None else None, size)
            return u.clone()

        def empty(*size, device=None, **kw):
            return shim._empty(*size, **kw)

        torch.Tensor.cuda = cuda
        torch.rand = rand
        torch.empty = empty
        return self

    def __exit__(self, *exc):
        self.torch.Tensor.cuda = self._cuda
        self.torch.rand = self._rand
        self.torch.empty = self._empty
        return False


def make_nbit(out: dict) -> None:
    import torch
    from ashkv.codecs.int2_dithered import DitheredINT2Codec
    from ashkv.codecs.nbit_dithered import DitheredNBitCodec

    def data(kind: str, n: int, g: torch.Generator) -> torch.Tensor:
        if kind == "normal":
            x = torch.randn(n, generator=g)
        elif kind == "outliers":  # 0.1% of entries x50 at seeded positions (the INT4 codec workload's distribution)
            x = torch.randn(n, generator=g)
            pos = torch.randperm(n, generator=g)[: max(1, n // 1000)]
            x[pos] *= 50.0
        elif kind == "headstd":  # per-row std ~U[0.5, 2] (the INT2 KV workload's distribution)
            x = torch.randn(n // 128, 128, generator=g) * (0.5 + 1.5 * torch.rand(n // 128, 1, generator=g))
            x = x.reshape(-1)
        elif kind == "wide":  # wide dynamic range: exercises the mean order and fp64 std
            x = torch.randn(n, generator=g) * torch.exp(torch.randn(n, generator=g) * 4.0)
        elif kind == "shifted":  # large common offset per group, small spread
            x = torch.randn(n // 32, 1, generator=g) * 100.0 + torch.randn(n // 32, 32, generator=g) * 0.05
            x = x.reshape(-1)
        elif kind == "special":  # constant groups, all-zero groups, tiny values, single spikes
            x = torch.randn(n, generator=g)
            x[0:32] = 0.0
            x[32:64] = 1.25
            x[64:96] = -3e-39
            x[96:128] = 1e-9 * torch.randn(32, generator=g)
            x[128:160] = 0.0; x[140] = 5.0
            x[160:192] = torch.arange(32, dtype=torch.float32)
            x[192:224] = -2.0; x[200] = 7.0; x[201] = -9.0
        else:
            raise ValueError(kind)
        return x

    cases = [
        # (codec, bits, sigma, hidden_dim, kind, n_elems, seed, trailing_bytes)
        ("nbit", 4, 3.0, 128, "outliers", 64 * 128, 0, 0),
        ("nbit", 4, 3.0, 128, "normal", 64 * 128, 1, 0),
        ("nbit", 4, 3.0, 128, "wide", 64 * 128, 2, 0),
        ("nbit", 4, 3.0, 128, "shifted", 64 * 128, 3, 0),
        ("nbit", 4, 3.0, 128, "special", 16 * 128, 4, 0),
        ("nbit", 2, 3.0, 128, "headstd", 64 * 128, 5, 0),
        ("nbit", 8, 3.0, 128, "outliers", 32 * 128, 6, 0),
        ("nbit", 4, 2.0, 64, "outliers", 64 * 64, 7, 0),
        ("nbit", 4, 1.0, 128, "normal", 16 * 128, 8, 0),
        ("nbit", 4, 3.0, 128, "normal", 5 * 128, 9, 6),   # ragged: 3 trailing bf16 values dropped
        ("nbit", 4, 3.0, 128, "normal", 0, 10, 100),      # shorter than one row -> empty
        ("int2", 2, 3.0, 128, "outliers", 64 * 128, 11, 0),
        ("int2", 2, 3.0, 128, "wide", 32 * 128, 12, 0),
        ("int2", 2, 3.0, 128, "special", 16 * 128, 13, 0),
    ]
    out["nbit_n_cases"] = np.array(len(cases))
    for ci, (codec_name, bits, sigma, hidden, kind, n, seed, trailing) in enumerate(cases):
        g = torch.Generator().manual_seed(1000 + seed)
        x = data(kind, n, g) if n else torch.zeros(0)
        xb = _bf16_bits(x)
        extra = (np.arange(trailing // 2, dtype=np.uint16) * 977 + 12345).astype(np.uint16)
        src_bits = np.concatenate([xb, extra]) if trailing else xb
        U = torch.rand(n, generator=torch.Generator().manual_seed(2000 + seed), dtype=torch.float32)
        if codec_name == "nbit":
            codec = DitheredNBitCodec(hidden_dim=hidden, group_size=32, sigma=sigma, bits=bits)
        else:
            codec = DitheredINT2Codec(hidden_dim=hidden)
        with _CpuShim() as shim:
            shim.U = U.view(n // hidden, hidden // 32, 32) if n else None
            blob = codec.encode(src_bits.tobytes())
            decoded = codec.decode(blob)
        pre = f"nbit_{ci}_"
        out[pre + "meta"] = np.array([bits, hidden, int(codec_name == "int2"), n, trailing], dtype=np.int64)
        out[pre + "sigma"] = np.array(sigma, dtype=np.float64)
        out[pre + "src"] = src_bits
        out[pre + "u"] = U.numpy()
        out[pre + "blob"] = np.frombuffer(blob, dtype=np.uint8).copy()
        out[pre + "decoded"] = np.frombuffer(decoded, dtype=np.uint8).copy()


def make_int8(out: dict) -> None:
    os.environ["TRITON_INTERPRET"] = "1"
    import torch
    from ashkv.codecs.int8 import _get_kernels

    enc, _ = _get_kernels()
    cases = [
        # (n_rows, row_len, scale dtype, data kind, seed)
        (64, 128, torch.float16, "normal", 0),
        (16, 1024, torch.float16, "normal", 1),
        (32, 256, torch.float16, "wide", 2),
        (8, 128, torch.float16, "special", 3),
        (8, 4096, torch.float16, "normal", 4),
    ]
    out["int8_n_cases"] = np.array(len(cases))
    for ci, (rows, L, sdt, kind, seed) in enumerate(cases):
        g = torch.Generator().manual_seed(3000 + seed)
        if kind == "normal":
            x = torch.randn(rows, L, generator=g) * 0.5 + 0.1
        elif kind == "wide":
            x = torch.randn(rows, L, generator=g) * torch.exp(torch.randn(rows, L, generator=g) * 2)
        else:
            x = torch.randn(rows, L, generator=g)
            x[0] = 0.0
            x[1] = 3.0
            x[2, 5] = 60000.0
            x[3] = torch.arange(L, dtype=torch.float32) / 10.0 - 6.0
        x16 = x.half()
        codes = torch.empty(rows, L, dtype=torch.int8)
        scales = torch.empty(rows, dtype=sdt)
        block = 128 if L % 128 == 0 else 64
        enc.fn[(rows,)](x16, codes, scales, rows, L, BLOCK_SIZE=block)
        pre = f"int8_{ci}_"
        out[pre + "meta"] = np.array([rows, L, int(sdt == torch.float16)], dtype=np.int64)
        out[pre + "src"] = x16.view(torch.int16).numpy().view(np.uint16).copy()
        out[pre + "codes"] = codes.numpy().copy()
        out[pre + "scales"] = scales.view(torch.int16).numpy().view(np.uint16).copy()


def make_policy(out: dict) -> None:
    from ashkv.compiler.runtime_builder import compile_controller
    from ashkv.contracts.config import ASHKVConfig
    from ashkv.runtime.controller import desired_tiers
    from ashkv.runtime.score import score_vectorized

    rng = np.random.default_rng(4242)
    n = 1 << 14
    T, S, N, P = (rng.random(n, dtype=np.float32) for _ in range(4))
    T[:8] = np.array([2.0, -1.0, np.nan, 0.0, 1.0, 0.5, np.inf, -np.inf], dtype=np.float32)
    cur = rng.integers(0, 4, n).astype(np.int8)
    cur[8:16] = np.array([4, 5, 4, 5, 0, 1, 2, 3], dtype=np.int8)
    cfg = ASHKVConfig()
    codec_keys = [(0, 1), (1, 0), (1, 2), (2, 1), (0, 2), (2, 0), (2, 3), (3, 2)]
    ctrl = compile_controller(cfg, {k: object() for k in codec_keys})
    closure = {name: c.cell_contents for name, c in zip(ctrl.__code__.co_freevars, ctrl.__closure__)}
    nc, nh = closure["next_colder"], closure["next_hotter"]
    R = score_vectorized(T, S, N, P, cfg.w_T, cfg.w_S, cfg.w_N, cfg.w_P)
    out["policy_T"], out["policy_S"], out["policy_N"], out["policy_P"] = T, S, N, P
    out["policy_cur"] = cur
    out["policy_R"] = R
    out["policy_next_colder"] = nc
    out["policy_next_hotter"] = nh
    out["policy_codec_keys"] = np.array(codec_keys, dtype=np.int64)
    pressures = np.array([0.0, 0.5, 0.7, 0.9, 0.95, 0.96, 0.97, 0.99, 1.0])
    out["policy_pressures"] = pressures
    for i, p in enumerate(pressures):
        out[f"policy_target_{i}"] = desired_tiers(R, cur, float(p), cfg.theta_high, cfg.theta_low,
                                                  cfg.delta, cfg.p_emergency, nc, nh)
    # Weights and thresholds that are not exactly representable (rounding probes).
    R2 = score_vectorized(T, S, N, P, 0.55, 0.15, 0.2, 0.1)
    out["policy_R2"] = R2
    out["policy_target_alt"] = desired_tiers(R2, cur, 0.963, 0.61, 0.29, 0.03, 0.9, nc, nh)


def make_xxh64(out: dict) -> None:
    from ashkv.codecs.checksum import checksum

    rng = np.random.default_rng(99)
    lengths = list(range(0, 80)) + [127, 128, 129, 255, 1000, 4096, 32768, 32768 + 7]
    blobs, digests = [], []
    for L in lengths:
        b = rng.integers(0, 256, L, dtype=np.uint8).tobytes()
        blobs.append(np.frombuffer(b, np.uint8))
        digests.append(checksum(b))
    out["xxh64_lengths"] = np.array(lengths, dtype=np.int64)
    out["xxh64_data"] = np.concatenate(blobs) if blobs else np.zeros(0, np.uint8)
    out["xxh64_digest"] = np.array(digests, dtype=np.uint64)


def make_fp8_int4(out: dict) -> None:
    import torch
    from ashkv.codecs.fp8 import FP8Codec
    from ashkv.codecs.int4 import INT4Codec

    assert not torch.cuda.is_available()
    allb = np.arange(65536, dtype=np.uint16)
    fp8 = FP8Codec()
    out["fp8_encode_all"] = np.frombuffer(fp8.encode(allb.tobytes()), np.uint8).copy()
    out["fp8_decode_all"] = np.frombuffer(fp8.decode(np.arange(256, dtype=np.uint8).tobytes()), np.uint16).copy()

    rng = np.random.default_rng(404)
    g = torch.Generator().manual_seed(404)
    cases = []
    cases.append((64, np.random.RandomState(42).randn(64 * 10).astype(np.float16).view(np.uint16)))
    cases.append((64, _bf16_bits(torch.randn(1000, generator=g) * 10)))
    cases.append((32, _bf16_bits(torch.randn(4096, generator=g))))
    x = torch.randn(8192, generator=g)
    x[torch.randint(0, 8192, (40,), generator=g)] *= 50
    cases.append((128, _bf16_bits(x)))
    cases.append((8, _bf16_bits(torch.randn(1024, generator=g) * 0.01)))
    cases.append((24, _bf16_bits(torch.randn(500, generator=g))))
    cases.append((7, _bf16_bits(torch.randn(70, generator=g))))
    cases.append((16, _bf16_bits(torch.randn(3, generator=g))))
    special = torch.zeros(16 * 10)
    special[0:16] = torch.randn(16, generator=g); special[3] = float("nan")
    special[16:32] = torch.randn(16, generator=g); special[20] = float("inf")
    special[32:48] = torch.randn(16, generator=g); special[40] = float("-inf")
    special[48:64] = torch.randn(16, generator=g) * 1e37; special[50] = 3.0e38; special[51] = -2.0e38
    special[64:80] = torch.randn(16, generator=g) * 1e-9
    special[80:96] = torch.tensor([7.0, 0.5, 1.5, 2.5, -0.5, -1.5, -2.5, 3.5, -3.5, 4.5, 5.5, -6.5, 6.5, 0.0,
                                   -0.0, -7.0])
    special[96:112] = torch.randn(16, generator=g) * 1e-39
    special[112:128] = -torch.rand(16, generator=g)
    special[128:144] = torch.full((16,), 1e-8)
    special[144:160] = torch.randn(16, generator=g) * 1e30
    cases.append((16, _bf16_bits(special)))
    raw = rng.integers(0, 65536, 4096, dtype=np.uint16)
    raw[(raw & 0x7F80) == 0x7F80] &= 0xBFFF   # keep most groups finite; a few NaN/inf remain below
    raw[[5, 700, 2100]] = [0x7FC1, 0x7F80, 0xFF80]
    cases.append((64, raw))
    blobs, inputs, gsz, decoded = [], [], [], []
    for gs, bits in cases:
        codec = INT4Codec(group_size=gs)
        blob = codec.encode(bits.astype(np.uint16).tobytes())
        inputs.append(bits.astype(np.uint16))
        blobs.append(np.frombuffer(blob, np.uint8).copy())
        decoded.append(np.frombuffer(codec.decode(blob), np.uint16).copy())
        gsz.append(gs)
    for i in range(len(cases)):
        out[f"int4_in_{i}"] = inputs[i]
        out[f"int4_blob_{i}"] = blobs[i]
        out[f"int4_dec_{i}"] = decoded[i]
    out["int4_group_size"] = np.array(gsz, dtype=np.int64)
    # decode of random blobs: scales over the whole bf16 range, random nibbles
    n_groups, gs = 256, 64
    sc = rng.integers(0, 65536, n_groups, dtype=np.uint16)
    sc[:4] = [0x7F80, 0xFF80, 0x7FC0, 0x0001]
    packed = rng.integers(0, 256, n_groups * gs // 2, dtype=np.uint8)
    import struct
    blob = struct.pack("<II", n_groups, n_groups * gs) + sc.tobytes() + packed.tobytes()
    out["int4_rand_blob"] = np.frombuffer(blob, np.uint8).copy()
    out["int4_rand_dec"] = np.frombuffer(INT4Codec(group_size=gs).decode(blob), np.uint16).copy()
    out["int4_empty_blob"] = np.frombuffer(INT4Codec().encode(b""), np.uint8).copy()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("ASHKV_REFERENCE"),
                    help="the reference source tree (default: $ASHKV_REFERENCE)")
    ap.add_argument("--out", default=str(HERE))
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference or set ASHKV_REFERENCE")
    sys.dont_write_bytecode = True
    sys.path.insert(0, args.reference)
    import ashkv  # noqa: F401  (the reference package)
    assert Path(ashkv.__file__).resolve().is_relative_to(Path(args.reference).resolve()), ashkv.__file__

    outdir = Path(args.out)
    for name, fn in (("nbit", make_nbit), ("int8", make_int8), ("policy", make_policy), ("xxh64", make_xxh64),
                     ("fp8_int4", make_fp8_int4)):
        d: dict = {}
        fn(d)
        np.savez_compressed(outdir / f"{name}.npz", **d)
        print(f"wrote {outdir / (name + '.npz')} ({(outdir / (name + '.npz')).stat().st_size} bytes)")


if __name__ == "__main__":
    main()
