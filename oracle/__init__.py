"""CPU oracle for the ASH-KV codec and policy path — TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, the arithmetic of the reference ASH-KV
implementation for the paths the CUDA kernels replace.  It is the checker:
only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s
``cpu_baseline`` / ``--impl reference`` legs import it.  The product
(``ashkv``) never imports, links or calls it.

Parity status: pinned.  ``tests/golden/`` holds fixtures produced by running
the reference's own Python code (N-bit/INT2 codecs with an injected dither,
score/controller, checksum) and its Triton INT8 kernel under the Triton
interpreter, and fixtures produced on a B200 by the reference's Triton INT8
kernels, its SGLang hooks, its simulator's attention mass and its N-bit codecs
run natively on CUDA (``tests/golden/make_golden_gpu.py``);
``tests/test_oracle_golden.py`` checks this oracle against all of them.  One
operation is restated up to ties: the Triton INT8 kernel divides with the
GPU's approximate ``div.full.f32``, the oracle exactly, and its tie mask marks
the elements where that can move a code by one.

Restated reference functions (paths relative to the ASH-KV source tree):

* ``int8_encode`` / ``int8_decode``   — ``ashkv/codecs/int8.py:50-81, 98-116``
* ``nbit_encode`` / ``nbit_decode``   — ``ashkv/codecs/nbit_dithered.py:43-167``,
  ``ashkv/codecs/int2_dithered.py:36-147``
* ``nbit_blob`` / ``nbit_parse_blob`` — blob layout, ``nbit_dithered.py:106-110``
* ``int8_blob``                       — ``ashkv/codecs/int8.py:179-182``
* ``xxh64``                           — ``ashkv/codecs/checksum.py:26-37``
* ``score``                           — ``ashkv/runtime/score.py:15-52``
* ``desired_tiers``                   — ``ashkv/runtime/controller.py:32-106``
* ``controller_tables``               — ``ashkv/compiler/runtime_builder.py:91-109``
* ``fp8_encode`` / ``fp8_decode``     — ``ashkv/codecs/fp8.py:32-79``
* ``int4_encode`` / ``int4_decode`` / ``int4_blob`` — ``ashkv/codecs/int4.py:38-112``
"""
from __future__ import annotations

import ctypes
import struct

import numpy as np

from . import build as _build

_LIB = None


def lib() -> ctypes.CDLL:
    """Load (building first if needed) the oracle's C library."""
    global _LIB
    if _LIB is None:
        path = _build.build()
        L = ctypes.CDLL(str(path))
        P = ctypes.c_void_p
        i64, i32, f32, u64 = ctypes.c_int64, ctypes.c_int32, ctypes.c_float, ctypes.c_uint64
        L.oracle_int8_encode.argtypes = [P, i32, i64, i32, i32, P, P, i32, P]
        L.oracle_int8_decode.argtypes = [P, P, i32, i64, i32, P, i32]
        L.oracle_nbit_encode.argtypes = [P, i64, i32, f32, P, P, P, P]
        L.oracle_nbit_decode.argtypes = [P, P, i64, i32, P, P, i64, P]
        L.oracle_xxh64.argtypes = [P, i64, u64]
        L.oracle_xxh64.restype = u64
        L.oracle_xxh64_items.argtypes = [P, i64, i64, i64, u64, P]
        L.oracle_philox4x32_10.argtypes = [P, P, P]
        L.oracle_philox_dither.argtypes = [i64, u64, u64, P]
        L.oracle_f32_to_bf16.argtypes = [f32]
        L.oracle_f32_to_bf16.restype = ctypes.c_uint16
        u16 = ctypes.c_uint16
        L.oracle_fp8_encode.argtypes = [P, i64, P]
        L.oracle_fp8_decode.argtypes = [P, i64, u16, P]
        L.oracle_int4_encode.argtypes = [P, i64, i32, i64, u16, P, P]
        L.oracle_int4_decode.argtypes = [P, P, i64, i32, u16, P]
        _LIB = L
    return _LIB


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


# --------------------------------------------------------------------- INT8
def int8_encode(x_bits: np.ndarray, row_len: int, src_fp16: bool = False, scale_fp16: bool = False,
                fp32_product: bool = False, with_ties: bool = False):
    """Rows of ``row_len`` bf16/fp16 values (uint16 bits) -> (int8 codes, uint16 scale bits)
    [, tie mask].  The oracle divides exactly; the reference's Triton kernel uses
    the GPU's approximate ``div.full.f32``.  The tie mask marks the elements whose
    exact quotient lies so close to a half-integer that the two can give codes
    one apart (see :func:`int8_codes_agree`)."""
    x = np.ascontiguousarray(x_bits, dtype=np.uint16).reshape(-1)
    n_rows = x.size // row_len
    codes = np.empty(n_rows * row_len, dtype=np.int8)
    scales = np.empty(n_rows, dtype=np.uint16)
    tie = np.zeros(n_rows * row_len, dtype=np.uint8)
    if n_rows:
        lib().oracle_int8_encode(_p(x), int(src_fp16), n_rows, row_len, int(fp32_product), _p(codes),
                                 _p(scales), int(scale_fp16), _p(tie))
    if with_ties:
        return codes.reshape(n_rows, row_len), scales, tie.reshape(n_rows, row_len).astype(bool)
    return codes.reshape(n_rows, row_len), scales


def int8_codes_agree(got: np.ndarray, want: np.ndarray, tie: np.ndarray) -> tuple[bool, int]:
    """(every code equals the oracle's, or differs by one at a tie-zone element; number of such ties)."""
    g = np.asarray(got).view(np.int8).astype(np.int16).reshape(-1)
    w = np.asarray(want).view(np.int8).astype(np.int16).reshape(-1)
    t = np.asarray(tie, dtype=bool).reshape(-1)
    diff = g != w
    ok = not np.any(diff & ~(t & (np.abs(g - w) == 1)))
    return ok, int(np.count_nonzero(diff))


def int8_decode(codes: np.ndarray, scales: np.ndarray, scale_fp16: bool = False,
                dst_fp16: bool = False) -> np.ndarray:
    c = np.ascontiguousarray(codes, dtype=np.int8)
    n_rows, row_len = c.shape
    s = np.ascontiguousarray(scales, dtype=np.uint16)
    out = np.empty(n_rows * row_len, dtype=np.uint16)
    if n_rows:
        lib().oracle_int8_decode(_p(c), _p(s), int(scale_fp16), n_rows, row_len, _p(out), int(dst_fp16))
    return out.reshape(n_rows, row_len)


def int8_blob(codes: np.ndarray, scales: np.ndarray) -> bytes:
    """INT8Codec blob: <I num_tokens> + bf16 scales + int8 codes."""
    return struct.pack("<I", codes.shape[0]) + scales.astype(np.uint16).tobytes() + codes.astype(np.int8).tobytes()


# --------------------------------------------------------------------- N-bit
def half_states(bits: int) -> float:
    return ((1 << bits) - 1) / 2.0


def nbit_encode(x_bits: np.ndarray, bits: int, dither: np.ndarray, sigma: float = 3.0):
    """Encode groups of 32 bf16 values.

    ``dither`` is the uniform ``U`` in [0, 1) (fp32, one per element).  Returns
    ``(scales uint16[n_groups], codes uint8[n_groups*32*bits/8],
    outlier_index int32[n], outlier_value uint16[n])`` with indices ascending.
    """
    x = np.ascontiguousarray(x_bits, dtype=np.uint16).reshape(-1)
    assert x.size % 32 == 0
    n_groups = x.size // 32
    d = np.ascontiguousarray(dither, dtype=np.float32).reshape(-1)
    assert d.size == x.size
    scales = np.empty(n_groups, dtype=np.uint16)
    codes = np.empty(n_groups * 32 * bits // 8, dtype=np.uint8)
    masks = np.empty(n_groups, dtype=np.uint32)
    if n_groups:
        lib().oracle_nbit_encode(_p(x), n_groups, bits, float(sigma), _p(d), _p(scales), _p(codes), _p(masks))
    bitpos = ((masks[:, None] >> np.arange(32, dtype=np.uint32)[None, :]) & 1).astype(bool).reshape(-1)
    idx = np.nonzero(bitpos)[0].astype(np.int32)
    vals = x[idx]
    return scales, codes, idx, vals


def nbit_decode(scales: np.ndarray, codes: np.ndarray, bits: int, idx: np.ndarray, vals: np.ndarray) -> np.ndarray:
    s = np.ascontiguousarray(scales, dtype=np.uint16)
    c = np.ascontiguousarray(codes, dtype=np.uint8)
    i = np.ascontiguousarray(idx, dtype=np.int32)
    v = np.ascontiguousarray(vals, dtype=np.uint16)
    n_groups = s.size
    out = np.empty(n_groups * 32, dtype=np.uint16)
    if n_groups:
        lib().oracle_nbit_decode(_p(s), _p(c), n_groups, bits, _p(i), _p(v), i.size, _p(out))
    return out


def nbit_blob(num_tokens: int, scales, codes, idx, vals) -> bytes:
    """Reference blob: <II tokens, n_out> + bf16 delta + int32 idx + bf16 vals + packed codes."""
    return (struct.pack("<II", num_tokens, len(idx)) + np.asarray(scales, np.uint16).tobytes()
            + np.asarray(idx, np.int32).tobytes() + np.asarray(vals, np.uint16).tobytes()
            + np.asarray(codes, np.uint8).tobytes())


def nbit_parse_blob(blob: bytes, hidden_dim: int = 128, group_size: int = 32):
    """Inverse of nbit_blob -> (num_tokens, scales, idx, vals, codes)."""
    num_tokens, n_out = struct.unpack("<II", blob[:8])
    n_scales = num_tokens * (hidden_dim // group_size)
    off = 8
    scales = np.frombuffer(blob, np.uint16, n_scales, off); off += 2 * n_scales
    idx = np.frombuffer(blob, np.int32, n_out, off); off += 4 * n_out
    vals = np.frombuffer(blob, np.uint16, n_out, off); off += 2 * n_out
    codes = np.frombuffer(blob, np.uint8, len(blob) - off, off)
    return num_tokens, scales, idx, vals, codes


def max_outliers_per_group(sigma: float, group: int = 32) -> int:
    """Upper bound on elements with |x-mu| > sigma*std in one group.

    m * sigma^2 < (group - 1) for the unbiased std, so m <= ceil((g-1)/sigma^2) - 1;
    one extra slot of margin covers rounding in the threshold.
    """
    if sigma <= 0:
        return group
    return int(min(group, np.floor((group - 1) / (sigma * sigma)) + 1))


# --------------------------------------------------------------------- hashes / RNG
def xxh64(data: bytes, seed: int = 0) -> int:
    buf = np.frombuffer(data, dtype=np.uint8) if len(data) else np.zeros(1, np.uint8)
    return int(lib().oracle_xxh64(_p(buf), len(data), seed))


def xxh64_items(data: np.ndarray, item_bytes: int, stride: int, n_items: int, seed: int = 0) -> np.ndarray:
    buf = np.ascontiguousarray(data).view(np.uint8).reshape(-1)
    out = np.empty(n_items, dtype=np.uint64)
    if n_items:
        lib().oracle_xxh64_items(_p(buf), n_items, item_bytes, stride, seed, _p(out))
    return out


def philox4x32_10(ctr, key) -> np.ndarray:
    c = np.asarray(ctr, dtype=np.uint32)
    k = np.asarray(key, dtype=np.uint32)
    out = np.empty(4, dtype=np.uint32)
    lib().oracle_philox4x32_10(_p(c), _p(k), _p(out))
    return out


def philox_dither(n: int, seed: int, offset: int = 0) -> np.ndarray:
    out = np.empty(n, dtype=np.float32)
    if n:
        lib().oracle_philox_dither(n, seed, offset, _p(out))
    return out


# --------------------------------------------------------------------- policy
NUM_TIERS = 6  # BF16, FP8, INT4, ARCHIVE, CPU, DISK
TIER_BF16, TIER_FP8, TIER_INT4 = 0, 1, 2


def score(T, S, N, P, w_T, w_S, w_N, w_P) -> np.ndarray:
    """R = clip(((wT*T + wS*S) + wN*N) + wP*P, 0, 1), each op one fp32 rounding."""
    n = len(T)
    if not (len(S) == len(N) == len(P) == n) or n == 0:
        return np.zeros(0, dtype=np.float32)
    R = np.float32(w_T) * T + np.float32(w_S) * S + np.float32(w_N) * N + np.float32(w_P) * P
    return np.clip(R, np.float32(0.0), np.float32(1.0))


def thresholds(pressure: float, theta_high: float, theta_low: float, delta: float,
               p_emergency: float) -> tuple[float, float]:
    """(promote_threshold, demote_threshold) in Python doubles."""
    boost = 0.0
    if pressure >= p_emergency:
        boost = min((pressure - p_emergency) * 2.0, 0.15)
    return theta_high + delta, (theta_low + boost) - delta


def desired_tiers(R, cur, pressure, theta_high, theta_low, delta, p_emergency, next_colder, next_hotter):
    n = len(R)
    if n == 0 or len(cur) != n:
        return np.asarray(cur).copy()
    up, down = thresholds(pressure, theta_high, theta_low, delta, p_emergency)
    tgt = np.array(cur, copy=True)
    pm = (R >= np.float32(up)) & (cur > TIER_BF16)
    tgt[pm] = next_hotter[cur[pm]]
    dm = (R <= np.float32(down)) & (cur < TIER_INT4)
    tgt[dm] = next_colder[cur[dm]]
    return tgt


def controller_tables(codec_keys) -> tuple[np.ndarray, np.ndarray]:
    """next_colder / next_hotter lookup tables from the codec table's (from, to) keys."""
    nc = np.arange(NUM_TIERS, dtype=np.int8)
    nh = np.arange(NUM_TIERS, dtype=np.int8)
    for i in range(NUM_TIERS - 1):
        nc[i] = i + 1
    for i in range(1, NUM_TIERS):
        nh[i] = i - 1
    keys = list(codec_keys)
    for src in range(NUM_TIERS):
        colder = [t for (s, t) in keys if s == src and t > src]
        if colder:
            nc[src] = min(colder)
        hotter = [t for (s, t) in keys if s == src and t < src]
        if hotter:
            nh[src] = max(hotter)
    return nc, nh


# --------------------------------------------------------------------- FP8
FP8_NAN_BF16_CUDA = 0x7FFF   # torch's CUDA float8 -> bf16 cast writes NaN as 0x7FFF
INT4_NAN_BF16_CPU = 0xFFFF   # torch's vectorised CPU float32 -> bf16 cast writes NaN as 0xFFFF


def fp8_encode(x_bits: np.ndarray) -> np.ndarray:
    """bf16 bits -> float8_e4m3fn bytes (torch's non-saturating cast)."""
    x = np.ascontiguousarray(x_bits, dtype=np.uint16).reshape(-1)
    out = np.empty(x.size, dtype=np.uint8)
    if x.size:
        lib().oracle_fp8_encode(_p(x), x.size, _p(out))
    return out


def fp8_decode(codes: np.ndarray, nan_bits: int = FP8_NAN_BF16_CUDA) -> np.ndarray:
    """float8_e4m3fn bytes -> bf16 bits."""
    c = np.ascontiguousarray(codes, dtype=np.uint8).reshape(-1)
    out = np.empty(c.size, dtype=np.uint16)
    if c.size:
        lib().oracle_fp8_decode(_p(c), c.size, nan_bits, _p(out))
    return out


# --------------------------------------------------------------------- INT4
def int4_encode(x_bits: np.ndarray, group_size: int = 64,
                nan_bits: int = INT4_NAN_BF16_CPU) -> tuple[np.ndarray, np.ndarray, int]:
    """bf16 bits -> (bf16 scale bits [n_groups], packed nibbles, num_values)."""
    x = np.ascontiguousarray(x_bits, dtype=np.uint16).reshape(-1)
    n_groups = -(-x.size // group_size)
    total = n_groups * group_size
    if total % 2:
        raise ValueError("padded value count must be even")
    scales = np.empty(n_groups, dtype=np.uint16)
    packed = np.empty(total // 2, dtype=np.uint8)
    if n_groups:
        lib().oracle_int4_encode(_p(x), x.size, group_size, n_groups, nan_bits, _p(scales), _p(packed))
    return scales, packed, total


def int4_decode(scales: np.ndarray, packed: np.ndarray, group_size: int = 64,
                nan_bits: int = INT4_NAN_BF16_CPU) -> np.ndarray:
    s = np.ascontiguousarray(scales, dtype=np.uint16).reshape(-1)
    p = np.ascontiguousarray(packed, dtype=np.uint8).reshape(-1)
    out = np.empty(s.size * group_size, dtype=np.uint16)
    if out.size:
        lib().oracle_int4_decode(_p(s), _p(p), s.size, group_size, nan_bits, _p(out))
    return out


def int4_blob(scales: np.ndarray, packed: np.ndarray, num_values: int) -> bytes:
    """INT4Codec blob (int4.py:74-75): <II num_groups, num_values> + bf16 scales + packed."""
    return struct.pack("<II", scales.size, num_values) + scales.astype(np.uint16).tobytes() + packed.tobytes()


# --------------------------------------------------------------------- page features
def attention_saliency(q, k, q_pos0=None, scale=None):
    """Attention mass per key as the reference simulator computes it
    (ashkv/tests/simulator.py:66-80): fp32 scores q.k / sqrt(head_dim), causal
    mask (key position <= query position), softmax over keys, summed over heads
    and queries.  q [n_q, heads_q, d], k [n_k, heads_kv, d] (torch, any float
    dtype; evaluated in fp32 on the CPU); query head h reads key head h // group."""
    import torch
    q = q.float().cpu()
    k = k.float().cpu()
    n_q, hq, d = q.shape
    n_k, hkv, _ = k.shape
    if q_pos0 is None:
        q_pos0 = n_k - n_q
    if scale is None:
        scale = 1.0 / (d ** 0.5)
    group = hq // hkv
    q_h = q.transpose(0, 1)                                  # [hq, n_q, d]
    k_h = k.transpose(0, 1).repeat_interleave(group, dim=0)  # [hq, n_k, d]
    scores = torch.matmul(q_h, k_h.transpose(-2, -1)) * scale
    qpos = torch.arange(n_q).view(-1, 1) + q_pos0
    kpos = torch.arange(n_k).view(1, -1)
    scores = scores.masked_fill(kpos > qpos, float("-inf"))
    attn = torch.softmax(scores, dim=-1)
    attn = torch.nan_to_num(attn, nan=0.0)   # rows with no visible key
    return attn.sum(dim=(0, 1))


def page_features(k, tokens_per_page, token_saliency=None):
    """(S, N) per page as the library defines them (numpy fp64 reference)."""
    import torch
    kf = k.float().cpu().reshape(k.shape[0], -1).double().numpy()
    n_k = kf.shape[0]
    n_pages = -(-n_k // tokens_per_page)
    delta = np.zeros(n_k)
    if n_k > 1:
        d = ((kf[1:] - kf[:-1]) ** 2).sum(1)
        nn = (kf[1:] ** 2).sum(1) + (kf[:-1] ** 2).sum(1)
        delta[1:] = np.where(nn > 0, 0.5 * d / np.where(nn > 0, nn, 1), 0.0)
    N = np.array([delta[p * tokens_per_page:(p + 1) * tokens_per_page].mean() for p in range(n_pages)])
    S = None
    if token_saliency is not None:
        s = np.asarray(token_saliency, dtype=np.float64)
        raw = np.array([s[p * tokens_per_page:(p + 1) * tokens_per_page].sum() for p in range(n_pages)])
        S = raw / raw.max() if raw.max() > 0 else raw * 0
    return S, N


# --------------------------------------------------------------------- tiered pages
# Page formats of the batched migration (ashkv_migrate_pages): a page is the
# bf16 values of its K rows then its V rows (E = 2 * T * row_len elements).
PAGE_BF16, PAGE_INT8, PAGE_FP8, PAGE_INT4, PAGE_NBIT4, PAGE_NBIT2 = 0, 1, 2, 3, 4, 5


def _int8_codes_offset(T: int) -> int:
    return (4 * T + 15) // 16 * 16


def page_encode(fmt: int, page_bits: np.ndarray, T: int, row_len: int, *, page_id: int = 0, seed: int = 0,
                sigma: float = 3.0, outlier_cap: int = 0):
    """bf16 page -> (slot bytes it defines, tie mask over those bytes, n_outliers).

    INT8: rows of ``row_len`` with fp16 scales (the hooks' row codec,
    ashkv/codecs/int8.py:50-81); FP8: FP8Codec (ashkv/codecs/fp8.py:32-79);
    INT4: INT4Codec, group 64 (ashkv/codecs/int4.py:38-75); NBIT4/NBIT2:
    DitheredNBitCodec / DitheredINT2Codec group arithmetic
    (ashkv/codecs/nbit_dithered.py:57-104) with U from Philox4x32-10(seed) at
    element offset page_id * E.  The tie mask marks INT8 code bytes that may be
    one apart (see int8_encode)."""
    x = np.ascontiguousarray(page_bits, dtype=np.uint16).reshape(-1)
    E = 2 * T * row_len
    assert x.size == E
    if fmt == PAGE_INT8:
        codes, scales, tie = int8_encode(x, row_len, scale_fp16=True, with_ties=True)
        c0 = _int8_codes_offset(T)
        out = np.zeros(c0 + E, np.uint8)
        out[:4 * T] = scales.view(np.uint8)
        out[c0:] = codes.view(np.uint8).reshape(-1)
        ties = np.zeros(out.size, bool)
        ties[c0:] = tie.reshape(-1)
        return out, ties, 0
    if fmt == PAGE_FP8:
        out = fp8_encode(x)
        return out, np.zeros(out.size, bool), 0
    if fmt == PAGE_INT4:
        scales, packed, _ = int4_encode(x, 64)
        out = np.concatenate([scales.view(np.uint8), packed])
        return out, np.zeros(out.size, bool), 0
    bits = 4 if fmt == PAGE_NBIT4 else 2
    U = philox_dither(E, seed, page_id * E)
    sc, codes, idx, vals = nbit_encode(x, bits, U, sigma)
    n_out = idx.size
    hdr = np.zeros(16, np.uint8)
    hdr[:4] = np.array([n_out if n_out <= outlier_cap else 0], np.uint32).view(np.uint8)
    ent = ((idx.astype(np.uint32) << 16) | vals.astype(np.uint32)).astype(np.uint32)
    body = [hdr, sc.view(np.uint8), codes]
    if n_out <= outlier_cap:
        body.append(ent.view(np.uint8))
    out = np.concatenate(body)
    return out, np.zeros(out.size, bool), n_out


def page_decode(fmt: int, slot: np.ndarray, T: int, row_len: int, *, outlier_cap: int = 0) -> np.ndarray:
    """Slot bytes -> bf16 page (the inverse codecs; INT8 decode as int8.py:98-116)."""
    s = np.ascontiguousarray(slot, dtype=np.uint8).reshape(-1)
    E = 2 * T * row_len
    if fmt == PAGE_INT8:
        c0 = _int8_codes_offset(T)
        scales = s[:4 * T].copy().view(np.uint16)
        codes = s[c0:c0 + E].copy().view(np.int8).reshape(2 * T, row_len)
        return int8_decode(codes, scales, scale_fp16=True).reshape(-1)
    if fmt == PAGE_FP8:
        return fp8_decode(s[:E])
    if fmt == PAGE_INT4:
        return int4_decode(s[:E // 32].copy().view(np.uint16), s[E // 32:E // 32 + E // 2], 64)
    bits = 4 if fmt == PAGE_NBIT4 else 2
    n_out = min(int(s[:4].copy().view(np.uint32)[0]), outlier_cap)
    d0, c0 = 16, 16 + E // 16
    e0 = c0 + E * bits // 8
    ent = s[e0:e0 + 4 * n_out].copy().view(np.uint32)
    return nbit_decode(s[d0:c0].copy().view(np.uint16), s[c0:e0], bits, (ent >> 16).astype(np.int32),
                       (ent & 0xFFFF).astype(np.uint16))
