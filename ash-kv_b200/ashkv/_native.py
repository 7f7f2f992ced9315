"""ctypes binding of libashkv_cuda.so (the C ABI declared in include/ashkv.h).

Every product code path that touches the codec arithmetic goes through the
functions below; there is no CPU fallback.  If the library is missing or
cannot be loaded, ``lib()`` raises :class:`NativeLibraryError`.

The wrappers accept torch CUDA tensors, check dtype/shape/alignment, pass raw
pointers plus torch's current stream, and raise :class:`KernelError` on a
non-zero status.  They never synchronise the device.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from ._build import LIB_PATH

OK, BAD_ARGUMENT, OUTLIER_OVERFLOW, LAUNCH_ERROR, TIMEOUT = 0, 1, 2, 3, 4
FLAG_OUTLIER_OVERFLOW = 0x1
FLAG_INDEX_RANGE = 0x2
DTYPE_BF16, DTYPE_FP16 = 0, 1
DITHER_TENSOR, DITHER_PHILOX = 0, 1
INT8_FP32_PRODUCT = 0x1
NBIT_GROUP = 32
NBIT_BUCKET_GROUPS = 32
NBIT_BUCKET_ELEMS = 1024

# name -> (restype, argtypes)
_P, _I32, _I64, _U32, _U64, _F32, _F64 = (ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_uint32,
                                         ctypes.c_uint64, ctypes.c_float, ctypes.c_double)
SIGNATURES: dict[str, tuple] = {
    "ashkv_version": (_I32, []),
    "ashkv_status_string": (ctypes.c_char_p, [_I32]),
    "ashkv_last_error": (ctypes.c_char_p, []),
    "ashkv_device_sm_count": (_I32, []),
    "ashkv_int8_encode_rows": (_I32, [_P, _I32, _I64, _I32, _I64, _P, _P, _I64, _P, _I32, _I32, _I64, _U32, _P]),
    "ashkv_int8_decode_rows": (_I32, [_P, _I64, _P, _I32, _I32, _I64, _I64, _I32, _P, _I32, _I64, _P, _P]),
    "ashkv_int8_encode_rows_layers": (_I32, [_P, _I32, _I32, _I64, _I32, _I64, _P, _P, _I64, _I64, _P, _I32, _I32,
                                             _I64, _I64, _U32, _P]),
    "ashkv_nbit_encode": (_I32, [_P, _I64, _I32, _F32, _I32, _P, _U64, _U64, _P, _P, _P, _P, _I32, _P, _P]),
    "ashkv_nbit_decode": (_I32, [_P, _P, _I64, _I32, _P, _P, _I32, _P, _P, _P]),
    "ashkv_nbit_outliers_flatten": (_I32, [_P, _P, _I32, _I64, _P, _P, _P, _P, _P]),
    "ashkv_nbit_decode_flat": (_I32, [_P, _P, _I64, _I32, _P, _P, _I64, _P, _P, _P]),
    "ashkv_xxh64_items": (_I32, [_P, _I64, _I64, _I64, _U64, _P, _P]),
    "ashkv_score": (_I32, [_P, _P, _P, _P, _I64, _F32, _F32, _F32, _F32, _P, _P]),
    "ashkv_desired_tiers": (_I32, [_P, _P, _I64, _F64, _F64, _F64, _F64, _F64, _P, _P, _P, _P]),
    "ashkv_policy_scratch_ints": (_I64, [_I64]),
    "ashkv_memcpy2d": (_I32, [_P, _I64, _P, _I64, _I64, _I64, _P]),
    "ashkv_fill32": (_I32, [_P, _I64, _U32, _P]),
    "ashkv_copy_rows_indexed": (_I32, [_P, _I64, _I64, _P, _I64, _P, _I64, _I64, _P, _I64, _I64, _I64, _I64, _P,
                                       _P]),
    "ashkv_policy_step_noalloc": (_I32, [_P, _P, _P, _P, _P, _I64, _F32, _F32, _F32, _F32, _F64, _F64, _F64, _F64,
                                         _F64, _P, _P, _P, _P, _P, _P, _P, _P]),
    "ashkv_int8_page_slot_bytes": (_I64, [_I32, _I32]),
    "ashkv_int8_encode_pages": (_I32, [_P, _P, _I32, _P, _P, _P, _P, _I32, _I32, _I32, _I64, _P, _I64, _I64, _P, _P,
                                       _P, _P, _P]),
    "ashkv_slots_commit": (_I32, [_P, _I32, _P, _P]),
    "ashkv_int8_decode_pages": (_I32, [_P, _P, _I32, _P, _P, _P, _P, _I32, _I32, _I32, _I64, _P, _I64, _I64, _P,
                                       _I32, _P, _P, _P, _P]),
    "ashkv_policy_step": (_I32, [_P, _P, _P, _P, _P, _I64, _F32, _F32, _F32, _F32, _F64, _F64, _F64, _F64,
                                 _F64, _P, _P, _P, _P, _P, _P, _P, _P, _P]),
    "ashkv_policy_step_device_pressure": (_I32, [_P, _P, _P, _P, _P, _I64, _F32, _F32, _F32, _F32, _P, _F64, _F64,
                                                 _F64, _F64, _P, _P, _P, _P, _P, _P, _P, _P, _P]),
    "ashkv_fp8_encode": (_I32, [_P, _I64, _P, _P]),
    "ashkv_fp8_decode": (_I32, [_P, _I64, _P, _P]),
    "ashkv_int4_group_count": (_I64, [_I64, _I32]),
    "ashkv_nbit_flatten_scratch_ints": (_I64, [_I64]),
    "ashkv_saliency_scratch_floats": (_I64, [_I32, _I64, _I64]),
    "ashkv_attention_saliency": (_I32, [_P, _P, _I32, _I32, _I32, _I64, _I64, _I64, _F32, _P, _P, _P, _P]),
    "ashkv_page_features": (_I32, [_P, _P, _I32, _I64, _I32, _P, _P, _P, _P]),
    "ashkv_int4_encode": (_I32, [_P, _I64, _I32, _P, _P, _P]),
    "ashkv_int4_decode": (_I32, [_P, _P, _I64, _I32, _P, _P]),
    "ashkv_page_slot_bytes": (_I64, [_I32, _I32, _I32, _I32]),
    "ashkv_migrate_pages": (_I32, [_P, _P, _P, _P, _P, _I64, _P, _P, _P, _I32, _P, _P, _I32, _I32, _I32, _I64, _P,
                                   _F32, _U64, _I32, _P, _P, _P]),
    "ashkv_release_slots": (_I32, [_P, _P, _I32, _P, _P, _P]),
}


class NativeLibraryError(RuntimeError):
    """libashkv_cuda.so is missing or could not be loaded."""


class KernelError(RuntimeError):
    """A library entry point returned a non-zero status."""

    def __init__(self, what: str, status: int, message: str):
        super().__init__(f"{what}: {message}")
        self.status = status


_LIB: Optional[ctypes.CDLL] = None


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            raise NativeLibraryError(
                f"{LIB_PATH} is not built; run `python -m ashkv._build` (needs nvcc) before using ashkv")
        try:
            L = ctypes.CDLL(str(LIB_PATH))
        except OSError as e:  # pragma: no cover - depends on the host
            raise NativeLibraryError(f"cannot load {LIB_PATH}: {e}") from e
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = L
    return _LIB


def status_string(status: int) -> str:
    return lib().ashkv_status_string(status).decode()


def check(status: int, what: str) -> None:
    if status != OK:
        msg = status_string(status)
        if status == LAUNCH_ERROR:
            msg += f" ({lib().ashkv_last_error().decode()})"
        raise KernelError(what, status, msg)


def stream_handle(device: Optional[torch.device] = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _require_cuda(*ts: Optional[torch.Tensor]) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("ashkv kernels take CUDA tensors")


def _dtype_tag(dt: torch.dtype) -> int:
    if dt == torch.bfloat16:
        return DTYPE_BF16
    if dt == torch.float16:
        return DTYPE_FP16
    raise TypeError(f"unsupported element type {dt}; expected bfloat16 or float16")


# --------------------------------------------------------------------------- INT8
def int8_encode_rows(src: torch.Tensor, codes: torch.Tensor, scales: torch.Tensor, *,
                     row_index: Optional[torch.Tensor] = None, scales_per_slot: int = 1,
                     scale_slot_stride: int = 2, fp32_product: bool = False) -> None:
    """Encode ``codes.shape[0]`` rows.  ``src`` is [rows_total, row_len] with unit
    inner stride (rows gathered by ``row_index`` if given); ``codes`` is
    [n_rows, row_len] int8/uint8 with unit inner stride; ``scales`` is the
    bf16/fp16 scale buffer addressed as in ashkv_int8_encode_rows."""
    _require_cuda(src, codes, scales, row_index)
    n_rows, row_len = codes.shape
    if src.dim() != 2 or src.shape[1] != row_len or src.stride(1) != 1 or codes.stride(1) != 1:
        raise ValueError("int8_encode_rows: src/codes must be 2-D [rows, row_len] with unit inner stride")
    if row_index is None and src.shape[0] < n_rows:
        raise ValueError("int8_encode_rows: src has fewer rows than codes")
    if row_index is not None and (row_index.dtype != torch.int64 or row_index.numel() != n_rows):
        raise ValueError("int8_encode_rows: row_index must be int64 with one entry per row")
    flags = INT8_FP32_PRODUCT if fp32_product else 0
    check(lib().ashkv_int8_encode_rows(
        src.data_ptr(), _dtype_tag(src.dtype), n_rows, row_len, src.stride(0), _ptr(row_index),
        codes.data_ptr(), codes.stride(0) * codes.element_size(),
        scales.data_ptr(), _dtype_tag(scales.dtype), scales_per_slot, scale_slot_stride, flags,
        stream_handle(src.device)), "int8_encode_rows")


def int8_encode_rows_layers(layer_ptrs: torch.Tensor, n_layers: int, src_dtype: torch.dtype, row_len: int,
                            src_row_stride: int, row_index: torch.Tensor, n_rows: int, codes_ptr: int,
                            codes_row_stride: int, layer_codes_offset: int, scales_ptr: int,
                            scales_per_slot: int, scale_slot_stride: int, layer_scales_offset: int,
                            device: torch.device) -> None:
    """``int8_encode_rows`` over ``n_layers`` layers in one launch (fp16 scales).  ``layer_ptrs``
    is an int64 CUDA tensor of 16-byte aligned layer base addresses; codes and scales are
    raw device addresses with per-layer byte offsets."""
    _require_cuda(layer_ptrs, row_index)
    if layer_ptrs.dtype != torch.int64 or layer_ptrs.numel() < n_layers:
        raise ValueError("int8_encode_rows_layers: layer_ptrs must hold n_layers int64 addresses")
    if row_index is None or row_index.dtype != torch.int64 or row_index.numel() != n_rows:
        raise ValueError("int8_encode_rows_layers: row_index must be int64 with one entry per row")
    check(lib().ashkv_int8_encode_rows_layers(
        layer_ptrs.data_ptr(), n_layers, _dtype_tag(src_dtype), n_rows, row_len, src_row_stride,
        row_index.data_ptr(), codes_ptr, codes_row_stride, layer_codes_offset, scales_ptr, DTYPE_FP16,
        scales_per_slot, scale_slot_stride, layer_scales_offset, 0, stream_handle(device)),
        "int8_encode_rows_layers")


def int8_decode_rows(codes: torch.Tensor, scales: torch.Tensor, dst: torch.Tensor, *,
                     row_index: Optional[torch.Tensor] = None, scales_per_slot: int = 1,
                     scale_slot_stride: int = 2) -> None:
    _require_cuda(codes, scales, dst, row_index)
    n_rows, row_len = codes.shape
    if dst.dim() != 2 or dst.shape[1] != row_len or dst.stride(1) != 1 or codes.stride(1) != 1:
        raise ValueError("int8_decode_rows: dst/codes must be 2-D [rows, row_len] with unit inner stride")
    if row_index is not None and (row_index.dtype != torch.int64 or row_index.numel() != n_rows):
        raise ValueError("int8_decode_rows: row_index must be int64 with one entry per row")
    check(lib().ashkv_int8_decode_rows(
        codes.data_ptr(), codes.stride(0) * codes.element_size(),
        scales.data_ptr(), _dtype_tag(scales.dtype), scales_per_slot, scale_slot_stride,
        n_rows, row_len, dst.data_ptr(), _dtype_tag(dst.dtype), dst.stride(0), _ptr(row_index),
        stream_handle(dst.device)), "int8_decode_rows")


# --------------------------------------------------------------------------- N-bit
def nbit_bucket_count(n_groups: int) -> int:
    return (n_groups + NBIT_BUCKET_GROUPS - 1) // NBIT_BUCKET_GROUPS


def nbit_encode(src: torch.Tensor, bits: int, sigma: float, scales: torch.Tensor, codes: torch.Tensor,
                bucket_counts: torch.Tensor, bucket_entries: torch.Tensor, bucket_cap: int,
                status: torch.Tensor, *, dither: Optional[torch.Tensor] = None, seed: int = 0,
                dither_offset: int = 0) -> None:
    """Encode ``src.numel() / 32`` groups (bf16, contiguous).  With ``dither``
    (fp32 U-0.5 per element) the TENSOR mode is used, else in-kernel Philox."""
    _require_cuda(src, scales, codes, bucket_counts, bucket_entries, status, dither)
    if src.dtype != torch.bfloat16 or not src.is_contiguous() or src.numel() % NBIT_GROUP:
        raise ValueError("nbit_encode: src must be contiguous bf16 with a multiple of 32 elements")
    n_groups = src.numel() // NBIT_GROUP
    if dither is not None and (dither.dtype != torch.float32 or dither.numel() != src.numel()
                               or not dither.is_contiguous()):
        raise ValueError("nbit_encode: dither must be contiguous fp32 with one value per element")
    nb = nbit_bucket_count(n_groups)
    if bucket_counts.numel() < nb or bucket_entries.numel() < nb * bucket_cap:
        raise ValueError("nbit_encode: bucket buffers too small")
    if scales.numel() < n_groups or codes.numel() * codes.element_size() < n_groups * 32 * bits // 8:
        raise ValueError("nbit_encode: output buffers too small")
    mode = DITHER_TENSOR if dither is not None else DITHER_PHILOX
    check(lib().ashkv_nbit_encode(
        src.data_ptr(), n_groups, bits, float(sigma), mode, _ptr(dither), seed & ((1 << 64) - 1),
        dither_offset, scales.data_ptr(), codes.data_ptr(), bucket_counts.data_ptr(),
        bucket_entries.data_ptr(), bucket_cap, status.data_ptr(), stream_handle(src.device)), "nbit_encode")


def nbit_decode(scales: torch.Tensor, codes: torch.Tensor, n_groups: int, bits: int, dst: torch.Tensor,
                status: torch.Tensor, bucket_counts: Optional[torch.Tensor] = None,
                bucket_entries: Optional[torch.Tensor] = None, bucket_cap: int = 0) -> None:
    _require_cuda(scales, codes, dst, status, bucket_counts, bucket_entries)
    if dst.numel() < n_groups * NBIT_GROUP or dst.dtype != torch.bfloat16:
        raise ValueError("nbit_decode: dst must be bf16 with n_groups*32 elements")
    check(lib().ashkv_nbit_decode(
        scales.data_ptr(), codes.data_ptr(), n_groups, bits, _ptr(bucket_counts), _ptr(bucket_entries),
        bucket_cap, dst.data_ptr(), status.data_ptr(), stream_handle(dst.device)), "nbit_decode")


def nbit_flatten_scratch_ints(n_buckets: int) -> int:
    return int(lib().ashkv_nbit_flatten_scratch_ints(n_buckets))


def nbit_outliers_flatten(bucket_counts: torch.Tensor, bucket_entries: torch.Tensor, bucket_cap: int,
                          n_buckets: int, offsets: torch.Tensor, out_index: torch.Tensor,
                          out_value: torch.Tensor, total: torch.Tensor) -> None:
    _require_cuda(bucket_counts, bucket_entries, offsets, out_index, out_value, total)
    if offsets.numel() < nbit_flatten_scratch_ints(n_buckets):
        raise ValueError("nbit_outliers_flatten: offsets needs nbit_flatten_scratch_ints(n_buckets) entries")
    check(lib().ashkv_nbit_outliers_flatten(
        bucket_counts.data_ptr(), bucket_entries.data_ptr(), bucket_cap, n_buckets, offsets.data_ptr(),
        out_index.data_ptr(), out_value.data_ptr(), total.data_ptr(), stream_handle(total.device)),
        "nbit_outliers_flatten")


def nbit_decode_flat(scales: torch.Tensor, codes: torch.Tensor, n_groups: int, bits: int,
                     out_index: Optional[torch.Tensor], out_value: Optional[torch.Tensor], n_outliers: int,
                     dst: torch.Tensor, status: torch.Tensor) -> None:
    _require_cuda(scales, codes, out_index, out_value, dst, status)
    if dst.numel() < n_groups * NBIT_GROUP or dst.dtype != torch.bfloat16:
        raise ValueError("nbit_decode_flat: dst must be bf16 with n_groups*32 elements")
    check(lib().ashkv_nbit_decode_flat(
        scales.data_ptr(), codes.data_ptr(), n_groups, bits, _ptr(out_index), _ptr(out_value), n_outliers,
        dst.data_ptr(), status.data_ptr(), stream_handle(dst.device)), "nbit_decode_flat")


# --------------------------------------------------------------------------- XXH64
def xxh64_items(data: torch.Tensor, n_items: int, item_bytes: int, item_stride: int, out: torch.Tensor,
                seed: int = 0) -> None:
    """One XXH64 digest per item into ``out`` (int64/uint64 tensor, bit pattern of the digest)."""
    _require_cuda(data, out)
    if out.numel() < n_items or out.element_size() != 8:
        raise ValueError("xxh64_items: out must hold n_items 64-bit values")
    check(lib().ashkv_xxh64_items(data.data_ptr(), n_items, item_bytes, item_stride, seed & ((1 << 64) - 1),
                                  out.data_ptr(), stream_handle(data.device)), "xxh64_items")


# --------------------------------------------------------------------------- FP8 / INT4
def _byte_view(t: torch.Tensor) -> torch.Tensor:
    if not t.is_contiguous():
        raise ValueError("ashkv codec buffers must be contiguous")
    return t


def fp8_encode(src: torch.Tensor, dst: torch.Tensor) -> None:
    """bf16 elements of ``src`` -> float8_e4m3fn bytes in ``dst`` (uint8 or float8_e4m3fn)."""
    _require_cuda(src, dst)
    _byte_view(src), _byte_view(dst)
    if src.dtype != torch.bfloat16:
        raise TypeError("fp8_encode takes bfloat16 input")
    n = src.numel()
    if dst.numel() * dst.element_size() < n:
        raise ValueError("fp8_encode: dst too small")
    check(lib().ashkv_fp8_encode(src.data_ptr(), n, dst.data_ptr(), stream_handle(src.device)), "fp8_encode")


def fp8_decode(src: torch.Tensor, dst: torch.Tensor) -> None:
    """float8_e4m3fn bytes of ``src`` -> bf16 elements of ``dst``."""
    _require_cuda(src, dst)
    _byte_view(src), _byte_view(dst)
    n = src.numel() * src.element_size()
    if dst.dtype != torch.bfloat16 or dst.numel() < n:
        raise ValueError("fp8_decode: dst must be bfloat16 with one element per code")
    check(lib().ashkv_fp8_decode(src.data_ptr(), n, dst.data_ptr(), stream_handle(src.device)), "fp8_decode")


def int4_group_count(n: int, group_size: int) -> int:
    return int(lib().ashkv_int4_group_count(n, group_size))


def int4_encode(src: torch.Tensor, group_size: int, scales: torch.Tensor, packed: torch.Tensor) -> None:
    """bf16 ``src`` (n elements, zero-padded to whole groups) -> bf16 ``scales`` + packed nibbles."""
    _require_cuda(src, scales, packed)
    _byte_view(src), _byte_view(scales), _byte_view(packed)
    if src.dtype != torch.bfloat16:
        raise TypeError("int4_encode takes bfloat16 input")
    n = src.numel()
    n_groups = -(-n // group_size) if group_size > 0 else 0
    if scales.numel() * scales.element_size() < 2 * n_groups or \
            packed.numel() * packed.element_size() < n_groups * group_size // 2:
        raise ValueError("int4_encode: output buffers too small")
    check(lib().ashkv_int4_encode(src.data_ptr(), n, group_size, scales.data_ptr(), packed.data_ptr(),
                                  stream_handle(src.device)), "int4_encode")


def int4_decode(scales: torch.Tensor, packed: torch.Tensor, n_groups: int, group_size: int,
                dst: torch.Tensor) -> None:
    _require_cuda(scales, packed, dst)
    _byte_view(scales), _byte_view(packed), _byte_view(dst)
    total = n_groups * group_size
    if dst.dtype != torch.bfloat16 or dst.numel() < total or \
            packed.numel() * packed.element_size() < total // 2 or scales.numel() * scales.element_size() < 2 * n_groups:
        raise ValueError("int4_decode: buffer sizes do not match n_groups * group_size")
    check(lib().ashkv_int4_decode(scales.data_ptr(), packed.data_ptr(), n_groups, group_size, dst.data_ptr(),
                                  stream_handle(dst.device)), "int4_decode")


# --------------------------------------------------------------------------- page features
def saliency_scratch_floats(heads_q: int, n_q: int, n_k: int) -> int:
    return int(lib().ashkv_saliency_scratch_floats(heads_q, n_q, n_k))


def attention_saliency(q: torch.Tensor, k: torch.Tensor, q_pos0: int, scale: float, scratch: torch.Tensor,
                       out: torch.Tensor, status: torch.Tensor) -> None:
    """q [n_q, heads_q, head_dim], k [n_k, heads_kv, head_dim] bf16 -> out[n_k] fp32 attention mass per key."""
    _require_cuda(q, k, scratch, out, status)
    if q.dtype != torch.bfloat16 or k.dtype != torch.bfloat16 or q.dim() != 3 or k.dim() != 3:
        raise TypeError("attention_saliency takes bf16 tensors [tokens, heads, head_dim]")
    if not (q.is_contiguous() and k.is_contiguous()):
        raise ValueError("attention_saliency: q and k must be contiguous")
    n_q, hq, d = q.shape
    n_k, hkv, dk = k.shape
    if dk != d:
        raise ValueError("q and k head_dim differ")
    if scratch.numel() < saliency_scratch_floats(hq, n_q, n_k) or out.numel() < n_k:
        raise ValueError("attention_saliency: scratch or out too small")
    check(lib().ashkv_attention_saliency(q.data_ptr(), k.data_ptr(), hq, hkv, d, n_q, n_k, q_pos0, scale,
                                         scratch.data_ptr(), out.data_ptr(), status.data_ptr(),
                                         stream_handle(q.device)), "attention_saliency")


def page_features(token_saliency: Optional[torch.Tensor], k: torch.Tensor, tokens_per_page: int,
                  s_raw: Optional[torch.Tensor], S: Optional[torch.Tensor], N: torch.Tensor) -> None:
    _require_cuda(token_saliency, k, s_raw, S, N)
    n_k = k.shape[0]
    row_len = k[0].numel() if n_k else 1
    n_pages = -(-n_k // tokens_per_page)
    if N.numel() < n_pages or (token_saliency is not None and (S.numel() < n_pages or s_raw.numel() < n_pages)):
        raise ValueError("page_features: outputs too small")
    check(lib().ashkv_page_features(_ptr(token_saliency), k.data_ptr(), row_len, n_k, tokens_per_page, _ptr(s_raw),
                                    _ptr(S), N.data_ptr(), stream_handle(k.device)), "page_features")


# --------------------------------------------------------------------------- policy
def _table(t) -> ctypes.Array:
    """Host int8[6] tier lookup table as a ctypes array (kept alive by the caller)."""
    import numpy as np
    a = np.asarray(t).reshape(-1)
    if a.size != 6:
        raise ValueError("tier lookup tables must have 6 entries (one per Tier)")
    return (ctypes.c_int8 * 6)(*[int(v) for v in a])


def _addr(arr: ctypes.Array) -> int:
    return ctypes.addressof(arr)


def score(T: torch.Tensor, S: torch.Tensor, N: torch.Tensor, P: torch.Tensor, w_T: float, w_S: float, w_N: float,
          w_P: float, R: torch.Tensor) -> None:
    _require_cuda(T, S, N, P, R)
    for t in (T, S, N, P, R):
        if t.dtype != torch.float32 or not t.is_contiguous():
            raise ValueError("score: float32 contiguous tensors expected")
    check(lib().ashkv_score(T.data_ptr(), S.data_ptr(), N.data_ptr(), P.data_ptr(), T.numel(), w_T, w_S, w_N,
                            w_P, R.data_ptr(), stream_handle(T.device)), "score")


def desired_tiers(R: torch.Tensor, cur: torch.Tensor, pressure: float, theta_high: float, theta_low: float,
                  delta: float, p_emergency: float, next_colder, next_hotter, target: torch.Tensor) -> None:
    _require_cuda(R, cur, target)
    if R.dtype != torch.float32 or cur.dtype != torch.int8 or target.dtype != torch.int8:
        raise ValueError("desired_tiers: R float32, cur/target int8 expected")
    nc, nh = _table(next_colder), _table(next_hotter)
    check(lib().ashkv_desired_tiers(R.data_ptr(), cur.data_ptr(), R.numel(), pressure, theta_high, theta_low,
                                    delta, p_emergency, _addr(nc), _addr(nh), target.data_ptr(),
                                    stream_handle(R.device)), "desired_tiers")


def policy_scratch_ints(n: int) -> int:
    return int(lib().ashkv_policy_scratch_ints(n))


def policy_step(T, S, N, P, cur, weights, pressure, theta_high: float, theta_low: float, delta: float,
                p_emergency: float, next_colder, next_hotter, R: Optional[torch.Tensor], target: torch.Tensor,
                demote_list: torch.Tensor, promote_list: torch.Tensor, counts: torch.Tensor,
                scratch: torch.Tensor) -> None:
    """``pressure`` is a Python float, or a one-element float32 CUDA tensor that the
    kernel reads on the device (no host read-back between a pressure all-reduce and
    the plan)."""
    _require_cuda(T, S, N, P, cur, R, target, demote_list, promote_list, counts, scratch)
    n = T.numel()
    if scratch.numel() < policy_scratch_ints(n) or demote_list.numel() < n or promote_list.numel() < n:
        raise ValueError("policy_step: list/scratch buffers too small")
    w_T, w_S, w_N, w_P = (float(w) for w in weights)
    nc, nh = _table(next_colder), _table(next_hotter)
    if isinstance(pressure, torch.Tensor):
        if not pressure.is_cuda or pressure.dtype != torch.float32 or pressure.numel() != 1:
            raise ValueError("policy_step: a device pressure must be a one-element float32 CUDA tensor")
        check(lib().ashkv_policy_step_device_pressure(
            T.data_ptr(), S.data_ptr(), N.data_ptr(), P.data_ptr(), cur.data_ptr(), n, w_T, w_S, w_N, w_P,
            pressure.data_ptr(), theta_high, theta_low, delta, p_emergency, _addr(nc), _addr(nh),
            _ptr(R), target.data_ptr(), demote_list.data_ptr(), promote_list.data_ptr(), counts.data_ptr(),
            scratch.data_ptr(), stream_handle(T.device)), "policy_step_device_pressure")
        return
    check(lib().ashkv_policy_step(
        T.data_ptr(), S.data_ptr(), N.data_ptr(), P.data_ptr(), cur.data_ptr(), n, w_T, w_S, w_N, w_P,
        pressure, theta_high, theta_low, delta, p_emergency, _addr(nc), _addr(nh),
        _ptr(R), target.data_ptr(), demote_list.data_ptr(), promote_list.data_ptr(), counts.data_ptr(),
        scratch.data_ptr(), stream_handle(T.device)), "policy_step")


# --------------------------------------------------------------------------- copies
def memcpy2d(dst_ptr: int, dst_pitch: int, src_ptr: int, src_pitch: int, width: int, height: int,
             device: Optional[torch.device] = None) -> None:
    """Pitched async copy on the current stream (host pointers should be pinned for async)."""
    check(lib().ashkv_memcpy2d(dst_ptr, dst_pitch, src_ptr, src_pitch, width, height, stream_handle(device)),
          "memcpy2d")


def fill32(t: torch.Tensor, value: int = 0) -> None:
    """Fill a contiguous CUDA tensor's bytes with a repeated 32-bit pattern on the current stream."""
    _require_cuda(t)
    if not t.is_contiguous():
        raise ValueError("fill32 needs a contiguous tensor")
    nbytes = t.numel() * t.element_size()
    check(lib().ashkv_fill32(t.data_ptr(), nbytes, value & 0xFFFFFFFF, stream_handle(t.device)), "fill32")


def copy_rows_indexed(dst_ptr: int, dst_row_stride: int, dst_sub_stride: int, dst_index: Optional[torch.Tensor],
                      dst_rows: int, src_ptr: int, src_row_stride: int, src_sub_stride: int,
                      src_index: Optional[torch.Tensor], src_rows: int, width: int, n_sub: int, n_rows: int,
                      device: torch.device, status: Optional[torch.Tensor] = None) -> None:
    """Indexed row gather/scatter between device memory and mapped page-locked host memory."""
    _require_cuda(dst_index, src_index, status)
    check(lib().ashkv_copy_rows_indexed(dst_ptr, dst_row_stride, dst_sub_stride, _ptr(dst_index), dst_rows,
                                        src_ptr, src_row_stride, src_sub_stride, _ptr(src_index), src_rows,
                                        width, n_sub, n_rows, _ptr(status), stream_handle(device)),
          "copy_rows_indexed")


POLICY_NOALLOC_MAX_PAGES = 4194304


def policy_step_noalloc(T, S, N, P, cur, weights, pressure: float, theta_high: float, theta_low: float,
                        delta: float, p_emergency: float, next_colder, next_hotter, R: Optional[torch.Tensor],
                        target: torch.Tensor, demote_list: torch.Tensor, promote_list: torch.Tensor,
                        counts: torch.Tensor) -> None:
    """``policy_step`` without a scratch buffer: for callers that cannot allocate device
    memory during a step.  The library keeps the per-block counts in a static device array
    (page tables up to POLICY_NOALLOC_MAX_PAGES entries); calls that overlap on the GPU race."""
    _require_cuda(T, S, N, P, cur, R, target, demote_list, promote_list, counts)
    n = T.numel()
    if demote_list.numel() < n or promote_list.numel() < n:
        raise ValueError("policy_step_noalloc: list buffers too small")
    w_T, w_S, w_N, w_P = (float(w) for w in weights)
    nc, nh = _table(next_colder), _table(next_hotter)
    check(lib().ashkv_policy_step_noalloc(
        T.data_ptr(), S.data_ptr(), N.data_ptr(), P.data_ptr(), cur.data_ptr(), n, w_T, w_S, w_N, w_P,
        pressure, theta_high, theta_low, delta, p_emergency, _addr(nc), _addr(nh), _ptr(R), target.data_ptr(),
        demote_list.data_ptr(), promote_list.data_ptr(), counts.data_ptr(), stream_handle(T.device)),
        "policy_step_noalloc")


# --------------------------------------------------------------------------- tiered pages
PAGE_NONE, PAGE_BF16, PAGE_INT8, PAGE_FP8, PAGE_INT4, PAGE_NBIT4, PAGE_NBIT2 = -1, 0, 1, 2, 3, 4, 5
MIGRATE_OK, MIGRATE_NO_SLOT, MIGRATE_BAD_PAGE, MIGRATE_PINNED, MIGRATE_SAME_TIER, MIGRATE_NO_CODEC, \
    MIGRATE_OVERFLOW = range(7)


class TierStoreDesc(ctypes.Structure):
    """ashkv_tier_store_t."""
    _fields_ = [("d_data", ctypes.c_void_p), ("slot_bytes", ctypes.c_int64), ("n_slots", ctypes.c_int32),
                ("format", ctypes.c_int32), ("d_free_stack", ctypes.c_void_p), ("d_free_top", ctypes.c_void_p)]


def page_slot_bytes(fmt: int, tokens_per_page: int, row_len: int, outlier_cap: int = 0) -> int:
    return int(lib().ashkv_page_slot_bytes(fmt, tokens_per_page, row_len, outlier_cap))


def migrate_pages(tier, pin, layer_id, token_start, page_slot, target, lst, count, layer_k_ptrs, layer_v_ptrs,
                  n_layers: int, tokens_per_page: int, row_len: int, row_stride: int, stores, sigma: float,
                  seed: int, outlier_cap: int, entry_status, released) -> None:
    """ashkv_migrate_pages; ``stores`` is a ctypes array of six TierStoreDesc (kept alive by the caller)."""
    _require_cuda(tier, pin, layer_id, token_start, page_slot, target, lst, count, entry_status, released)
    check(lib().ashkv_migrate_pages(
        tier.data_ptr(), _ptr(pin), layer_id.data_ptr(), token_start.data_ptr(), page_slot.data_ptr(), tier.numel(),
        target.data_ptr(), lst.data_ptr(), count.data_ptr(), lst.numel(), layer_k_ptrs.data_ptr(),
        layer_v_ptrs.data_ptr(), n_layers, tokens_per_page, row_len, row_stride, ctypes.addressof(stores),
        float(sigma), int(seed) & 0xFFFFFFFFFFFFFFFF, outlier_cap, entry_status.data_ptr(), released.data_ptr(),
        stream_handle(tier.device)), "migrate_pages")


def release_slots(released, count, max_entries: int, stores, status=None) -> None:
    _require_cuda(released, count, status)
    check(lib().ashkv_release_slots(released.data_ptr(), count.data_ptr(), max_entries, ctypes.addressof(stores),
                                    _ptr(status), stream_handle(released.device)), "release_slots")
