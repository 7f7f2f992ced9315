"""Generate the GPU-side golden fixtures by running the reference ASH-KV code on a CUDA GPU.

The reference's Triton INT8 kernels, its SGLang hooks and its simulator run
only on a GPU, so these fixtures are produced on a B200 from a copy of the
reference package (``oracle/reference_copy.py`` puts it in ``oracle/_ref``):

    python tests/golden/make_golden_gpu.py --reference oracle/_ref --out <dir>

The reference is imported as the ``ashkv`` package from ``--reference``; this
script never imports this repository's own ``ashkv``.  It writes:

* ``int8_bf16.npz`` — ``_int8_encode_kernel`` / ``_int8_decode_kernel``
  (``ashkv/codecs/int8.py:50-116``) on bf16 rows of 8, 24, 128, 1000 and 1024
  elements with bf16 and fp16 scale buffers (normal rows over a wide range of
  magnitudes; rows with NaN, +-inf, subnormals, zeros, values near the bf16
  maximum, near-.5 quotients and absmax below the 1e-8 floor), run through the
  autotuner and through each of its nine configurations; decode of every
  int8 code under bf16 and fp16 scales (random bit patterns plus specials).
* ``hooks_int8.npz`` — ``SGLangHooks.demote_hook`` / ``promote_hook``
  (``ashkv/adapters/sglang/hooks.py:51-245``) on mock pools: the host slots
  written by demote and the device rows restored by promote.
* ``saliency.npz`` — the simulator's per-key attention mass
  (``ashkv/tests/simulator.py:66-74``), captured at its ``torch.topk`` call,
  with the simulator's own q and k.
* ``nbit_cuda.npz`` — ``DitheredNBitCodec(bits=4)`` and ``DitheredINT2Codec``
  run natively on CUDA (their production device), with the ``torch.rand``
  output each encode drew recorded next to the blob.

Inputs are seeded synthetic data.
"""
from __future__ import annotations

import argparse
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent

INT8_ROW_LENS = (8, 24, 128, 1000, 1024)
TRITON_CONFIGS = [(b, w) for b in (64, 128, 256) for w in (2, 4, 8)]


def _bits16(t) -> np.ndarray:
    import torch
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16).copy()


def _bf16_from_bits(bits: np.ndarray):
    import torch
    return torch.from_numpy(bits.astype(np.uint16).view(np.int16)).view(torch.bfloat16)


def _f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    import torch
    return _bits16(torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(torch.bfloat16))


def int8_rows(L: int, rng: np.random.Generator) -> np.ndarray:
    """bf16 bit patterns [rows, L]: normal rows plus special rows."""
    n_norm = max(32, 32768 // L)
    mag = np.exp2(rng.uniform(-40, 40, size=(n_norm, 1)))
    norm = _f32_to_bf16_bits(rng.standard_normal((n_norm, L)).astype(np.float32) * mag)
    special = []

    def row(vals):
        return _f32_to_bf16_bits(np.asarray(vals, dtype=np.float32)).reshape(1, L)

    base = rng.standard_normal(L).astype(np.float32)
    special.append(np.zeros((1, L), np.uint16))                       # all zero
    r = base.copy(); r[rng.integers(0, L)] = np.nan; special.append(row(r))  # one NaN
    special.append(np.full((1, L), 0x7FC0, np.uint16))                # all NaN
    r = base.copy(); r[0] = np.inf; special.append(row(r))            # +inf (absmax inf)
    r = base.copy(); r[-1] = -np.inf; special.append(row(r))          # -inf
    r = base.copy(); r[0] = np.inf; r[1 % L] = np.nan; special.append(row(r))
    sub = rng.integers(1, 0x80, size=(1, L)).astype(np.uint16)        # bf16 subnormals
    sub[0, ::2] |= 0x8000
    special.append(sub)
    special.append(row(base * 1e-39))                                  # mostly subnormal after rounding
    special.append(row(base * 1e-12))                                  # absmax below the 1e-8 floor
    special.append(row(base * 3e36))                                   # x*127 overflows bf16
    big = np.full(L, 3.3e38, np.float32); big[::3] *= -1; special.append(row(big))
    # near-.5 quotients: bf16(v*127)/am close to k + 0.5 for an absmax am at element 0
    for am in (1.0, 0.7734375, 3.140625, 1.0e-3, 5.0e4):
        t = (np.arange(L) % 254 - 126.5 + 0.5 * (np.arange(L) % 2)).astype(np.float64)
        v = (t + 0.5) * am / 127.0
        vb = _f32_to_bf16_bits(v.astype(np.float32)).astype(np.int32)
        step = rng.integers(-2, 3, size=L)
        vb = np.where(vb & 0x7FFF, vb + step, vb).astype(np.uint16)
        vb[0] = _f32_to_bf16_bits(np.array([am], np.float32))[0]
        special.append(vb.reshape(1, L))
    return np.concatenate([norm] + special, axis=0)


def make_int8(out: dict) -> None:
    import torch
    from ashkv.codecs.int8 import _get_kernels  # the reference's Triton kernels
    enc, dec = _get_kernels()
    dev = torch.device("cuda")
    rng = np.random.default_rng(20260)
    mismatched_configs = []
    for L in INT8_ROW_LENS:
        bits = int8_rows(L, rng)
        n = bits.shape[0]
        src = _bf16_from_bits(bits).view(n, L).to(dev)
        out[f"enc_in_L{L}"] = bits
        for sname, sdt in (("bf16", torch.bfloat16), ("fp16", torch.float16)):
            codes = torch.empty((n, L), dtype=torch.int8, device=dev)
            scales = torch.empty((n,), dtype=sdt, device=dev)
            enc[(n,)](src, codes, scales, n, L)  # autotuned (production) path
            torch.cuda.synchronize()
            c_auto, s_auto = codes.cpu().numpy().copy(), _bits16(scales)
            out[f"enc_codes_L{L}_{sname}"] = c_auto.view(np.int8)
            out[f"enc_scales_L{L}_{sname}"] = s_auto
            for (b, w) in TRITON_CONFIGS:
                codes.fill_(0); scales.fill_(0)
                enc.fn[(n,)](src, codes, scales, n, L, BLOCK_SIZE=b, num_warps=w)
                torch.cuda.synchronize()
                if not (np.array_equal(codes.cpu().numpy(), c_auto) and np.array_equal(_bits16(scales), s_auto)):
                    mismatched_configs.append(f"enc L={L} {sname} BLOCK={b} warps={w}")
    # decode: every code under many scales
    L = 256
    codes_row = (np.arange(256) - 128).astype(np.int8)
    for sname, sdt in (("bf16", torch.bfloat16), ("fp16", torch.float16)):
        sc = rng.integers(0, 65536, size=2048, dtype=np.uint16)
        sc[:8] = [0x0000, 0x8000, 0x0001, 0x7F80 if sname == "bf16" else 0x7C00,
                  0x7FC0 if sname == "bf16" else 0x7E00, 0x3F80 if sname == "bf16" else 0x3C00,
                  0x7F7F if sname == "bf16" else 0x7BFF, 0x0080 if sname == "bf16" else 0x0400]
        n = sc.size
        c = torch.from_numpy(np.tile(codes_row, (n, 1))).to(dev)
        s = torch.from_numpy(sc.view(np.int16)).view(sdt).to(dev)
        o = torch.empty((n, L), dtype=torch.bfloat16, device=dev)
        dec[(n,)](c, s, o, n, L)
        torch.cuda.synchronize()
        ref = _bits16(o)
        for (b, w) in TRITON_CONFIGS:
            o.zero_()
            dec.fn[(n,)](c, s, o, n, L, BLOCK_SIZE=b, num_warps=w)
            torch.cuda.synchronize()
            if not np.array_equal(_bits16(o), ref):
                mismatched_configs.append(f"dec {sname} BLOCK={b} warps={w}")
        out[f"dec_scales_{sname}"] = sc
        out[f"dec_out_{sname}"] = ref.reshape(n, L)
    out["dec_codes_row"] = codes_row
    out["row_lens"] = np.array(INT8_ROW_LENS, np.int64)
    out["config_mismatches"] = np.array(mismatched_configs, dtype=object).astype(str)
    print(f"int8: configs disagreeing with the autotuned output: {mismatched_configs or 'none'}")


class _DevPool:
    def __init__(self, layers, cap, H, D, rng):
        import torch
        self.head_num, self.head_dim, self.layer_num = H, D, layers
        x = rng.standard_normal((2, layers, cap, H, D)).astype(np.float32)
        x[rng.random(x.shape) < 0.002] *= 40.0
        t = torch.from_numpy(x).to(torch.bfloat16).cuda()
        self.k_buffer = [t[0, l].contiguous() for l in range(layers)]
        self.v_buffer = [t[1, l].contiguous() for l in range(layers)]


class _HostPool:
    def __init__(self, layers, cap, H, D):
        import torch
        self.k_buffer = torch.zeros((cap, layers, H, D), dtype=torch.bfloat16)
        self.v_buffer = torch.zeros((cap, layers, H, D), dtype=torch.bfloat16)


def make_hooks(out: dict) -> None:
    import torch
    from ashkv.adapters.sglang.hooks import SGLangHooks
    rng = np.random.default_rng(20261)
    cases = [  # (layers, device capacity, host capacity, H, D, n tokens, host indices contiguous)
        (2, 96, 80, 8, 128, 40, True),
        (3, 64, 64, 1, 128, 33, False),
        (2, 48, 40, 4, 64, 17, False),
    ]
    for i, (layers, cap, hcap, H, D, n, contiguous) in enumerate(cases):
        dp = _DevPool(layers, cap, H, D, rng)
        hp = _HostPool(layers, hcap, H, D)
        dev_idx = np.sort(rng.choice(cap, size=n, replace=False)).astype(np.int64)
        host_idx = (np.arange(n) + 5 if contiguous else rng.choice(hcap, size=n, replace=False)).astype(np.int64)
        out[f"case{i}_shape"] = np.array([layers, cap, hcap, H, D, n], np.int64)
        out[f"case{i}_dev_k"] = np.stack([_bits16(t) for t in dp.k_buffer])
        out[f"case{i}_dev_v"] = np.stack([_bits16(t) for t in dp.v_buffer])
        out[f"case{i}_dev_idx"] = dev_idx
        out[f"case{i}_host_idx"] = host_idx
        hooks = SGLangHooks(codec_name="int8_default")
        hooks.stats_file = str(Path(out["_tmp"]) / f"stats{i}.json")
        d_idx = torch.from_numpy(dev_idx).cuda()
        h_idx = torch.from_numpy(host_idx)
        assert hooks.demote_hook(dp, hp, h_idx, d_idx, "MHA")
        torch.cuda.synchronize()
        out[f"case{i}_host_k"] = _bits16(hp.k_buffer[h_idx])   # [n, layers, H, D] slot bytes as u16
        out[f"case{i}_host_v"] = _bits16(hp.v_buffer[h_idx])
        for t in dp.k_buffer + dp.v_buffer:
            t.zero_()
        for l in range(layers):
            assert hooks.promote_hook(dp, hp, h_idx, d_idx, l, "MHA")
        torch.cuda.synchronize()
        out[f"case{i}_prom_k"] = np.stack([_bits16(t[d_idx]) for t in dp.k_buffer])
        out[f"case{i}_prom_v"] = np.stack([_bits16(t[d_idx]) for t in dp.v_buffer])
    out["n_cases"] = np.array(len(cases), np.int64)


def make_saliency(out: dict) -> None:
    import torch
    from ashkv.tests.simulator import E2ESimulator
    cases = [(512, 8, 64), (384, 4, 128)]
    for i, (S, H, D) in enumerate(cases):
        torch.manual_seed(1000 + i)
        sim = E2ESimulator(seq_len=S, head_num=H, head_dim=D, gpu_capacity=S // 2)
        hidden = torch.randn((S, H * D), dtype=torch.bfloat16, device="cuda")
        with torch.no_grad():
            k_full = sim.k_proj(hidden).view(S, H, D)
            v_full = sim.v_proj(hidden).view(S, H, D)
        got = {}
        h = sim.q_proj.register_forward_hook(lambda m, a, o: got.setdefault("q", o.detach().clone()))
        orig_topk = torch.topk

        def topk(t, *a, **kw):
            got.setdefault("saliency", t.detach().clone())
            return orig_topk(t, *a, **kw)

        torch.topk = topk
        try:
            with torch.no_grad():
                sim.run_int8_via_hooks(hidden, k_full, v_full)
        finally:
            torch.topk = orig_topk
            h.remove()
        torch.cuda.synchronize()
        out[f"case{i}_q"] = _bits16(got["q"].view(S, H, D))
        out[f"case{i}_k"] = _bits16(k_full)
        out[f"case{i}_saliency"] = got["saliency"].float().cpu().numpy()
        out[f"case{i}_shape"] = np.array([S, H, D], np.int64)
    out["n_cases"] = np.array(len(cases), np.int64)


def make_nbit_cuda(out: dict) -> None:
    import torch
    from ashkv.codecs.int2_dithered import DitheredINT2Codec
    from ashkv.codecs.nbit_dithered import DitheredNBitCodec
    rng = np.random.default_rng(20262)
    x = rng.standard_normal(512 * 128).astype(np.float32)
    x[rng.random(x.size) < 0.001] *= 50.0
    bits = _f32_to_bf16_bits(x)
    out["input"] = bits
    for name, codec in (("nbit4", DitheredNBitCodec(bits=4)), ("int2", DitheredINT2Codec())):
        drawn = []
        orig_rand = torch.rand

        def rand(*a, **kw):
            u = orig_rand(*a, **kw)
            drawn.append(u.detach().float().cpu().numpy().copy())
            return u

        torch.rand = rand
        try:
            blob = codec.encode(bits.tobytes())
        finally:
            torch.rand = orig_rand
        assert len(drawn) == 1, len(drawn)
        out[f"{name}_uniform"] = drawn[0].reshape(-1)
        out[f"{name}_blob"] = np.frombuffer(blob, np.uint8).copy()
        out[f"{name}_decoded"] = np.frombuffer(codec.decode(blob), np.uint16).copy()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="directory holding the reference's ashkv/ package")
    ap.add_argument("--out", default=str(HERE))
    ap.add_argument("--only", default="", help="comma-separated subset of int8,hooks,saliency,nbit_cuda")
    args = ap.parse_args()
    sys.dont_write_bytecode = True
    sys.path.insert(0, str(Path(args.reference).resolve()))
    import torch
    import triton
    import ashkv  # noqa: F401  (the reference package)
    assert Path(ashkv.__file__).resolve().is_relative_to(Path(args.reference).resolve()), ashkv.__file__
    assert torch.cuda.is_available(), "the reference's Triton kernels need a CUDA GPU"
    outdir = Path(args.out)
    outdir.mkdir(parents=True, exist_ok=True)
    meta = {"torch": torch.__version__, "triton": triton.__version__, "gpu": torch.cuda.get_device_name(0)}
    only = {s for s in args.only.split(",") if s}
    for name, fn in (("int8_bf16", make_int8), ("hooks_int8", make_hooks), ("saliency", make_saliency),
                     ("nbit_cuda", make_nbit_cuda)):
        key = name.split("_")[0] if name != "nbit_cuda" else "nbit_cuda"
        if only and key not in only and name not in only:
            continue
        d: dict = {"_tmp": str(outdir)}
        fn(d)
        d.pop("_tmp")
        for k, v in meta.items():
            d[f"meta_{k}"] = np.array(v)
        np.savez_compressed(outdir / f"{name}.npz", **d)
        print(f"wrote {outdir / (name + '.npz')} ({(outdir / (name + '.npz')).stat().st_size} bytes)")


if __name__ == "__main__":
    main()
