"""INT8 per-row absmax codec on sm_100a.

Drop-in for ``INT8Codec`` (ashkv/codecs/int8.py:135-225 of the reference):
same constructor (``hidden_dim``), same blob
``<I num_tokens> + bf16 scale[num_tokens] + int8 code[num_tokens*hidden_dim]``,
same empty/short-input behaviour and the same ``checksum``.  The Triton
``_int8_encode_kernel``/``_int8_decode_kernel`` it used are replaced by
``ashkv_int8_encode_rows``/``ashkv_int8_decode_rows``.

``encode_rows``/``decode_rows`` are the device-resident entry points used by
the SGLang hooks and the batched migrate path.
"""
from __future__ import annotations

import struct
from typing import Optional

import torch

from .. import _native, _staging
from .checksum import checksum


def encode_rows(src: torch.Tensor, *, scale_dtype: torch.dtype = torch.bfloat16,
                codes: Optional[torch.Tensor] = None, scales: Optional[torch.Tensor] = None,
                fp32_product: bool = False) -> tuple[torch.Tensor, torch.Tensor]:
    """Encode a CUDA tensor [n_rows, row_len] (bf16/fp16) -> (int8 codes, scales)."""
    n_rows, row_len = src.shape
    if codes is None:
        codes = torch.empty((n_rows, row_len), dtype=torch.int8, device=src.device)
    if scales is None:
        scales = torch.empty((n_rows,), dtype=scale_dtype, device=src.device)
    _native.int8_encode_rows(src, codes, scales, fp32_product=fp32_product)
    return codes, scales


def decode_rows(codes: torch.Tensor, scales: torch.Tensor, *, out_dtype: torch.dtype = torch.bfloat16,
                out: Optional[torch.Tensor] = None) -> torch.Tensor:
    n_rows, row_len = codes.shape
    if out is None:
        out = torch.empty((n_rows, row_len), dtype=out_dtype, device=codes.device)
    _native.int8_decode_rows(codes, scales, out)
    return out


class _RowKernel:
    """A launcher with the call shape of the reference's Triton INT8 kernels.

    ``kernel[grid](a, b, c, num_tokens, hidden_dim)`` runs one row per program
    of ``grid`` (as the Triton kernel does: it never reads ``num_tokens``) over
    contiguous buffers addressed as ``row * hidden_dim + i``.  Triton meta
    arguments (``BLOCK_SIZE``, ``num_warps``) are accepted and ignored.
    """

    def __init__(self, launch):
        self._launch = launch

    def __getitem__(self, grid):
        rows = int(grid[0] if isinstance(grid, (tuple, list)) else grid)

        def run(a, b, c, num_tokens, hidden_dim, **_meta):
            self._launch(rows, int(hidden_dim), a, b, c)
        return run


def _flat_rows(t: torch.Tensor, rows: int, L: int, what: str) -> torch.Tensor:
    if not t.is_contiguous():
        raise ValueError(f"{what} must be contiguous (the kernel addresses it as row * hidden_dim + i)")
    flat = t.view(-1)
    if flat.numel() < rows * L:
        raise ValueError(f"{what} holds {flat.numel()} elements, fewer than {rows} rows of {L}")
    return flat[: rows * L].view(rows, L)


def _flat_scales(t: torch.Tensor, rows: int) -> torch.Tensor:
    if not t.is_contiguous() or t.numel() < rows:
        raise ValueError(f"scale buffer must be contiguous with at least {rows} entries")
    return t.view(-1)


def _launch_encode(rows: int, L: int, src: torch.Tensor, codes: torch.Tensor, scales: torch.Tensor) -> None:
    if rows == 0:
        return
    _native.int8_encode_rows(_flat_rows(src, rows, L, "input"), _flat_rows(codes, rows, L, "code buffer"),
                             _flat_scales(scales, rows))


def _launch_decode(rows: int, L: int, codes: torch.Tensor, scales: torch.Tensor, dst: torch.Tensor) -> None:
    if rows == 0:
        return
    _native.int8_decode_rows(_flat_rows(codes, rows, L, "code buffer"), _flat_scales(scales, rows),
                             _flat_rows(dst, rows, L, "output"))


_KERNELS = (_RowKernel(_launch_encode), _RowKernel(_launch_decode))


def _get_kernels():
    """(encode, decode) launchers in the call shape of ``_get_kernels()`` of the
    reference (ashkv/codecs/int8.py:27-120), so code written against the Triton
    kernels — ``encode[grid](src, int8_out, scale_out, num_tokens, hidden_dim)``
    and ``decode[grid](int8_in, scale_in, out, num_tokens, hidden_dim)`` — runs
    on ``ashkv_int8_encode_rows`` / ``ashkv_int8_decode_rows``.  Inputs are bf16
    or fp16 rows; scale buffers bf16 or fp16 (one per row, flat index = row)."""
    return _KERNELS


class INT8Codec:
    """INT8 codec with one bf16 absmax scale per ``hidden_dim``-element row."""

    __slots__ = ("_encode_calls", "_decode_calls", "_hidden_dim")

    def __init__(self, hidden_dim: int = 128) -> None:
        self._encode_calls = 0
        self._decode_calls = 0
        self._hidden_dim = hidden_dim

    def encode(self, source_bytes: bytes) -> bytes:
        self._encode_calls += 1
        if not source_bytes:
            return struct.pack("<I", 0)
        _staging.check_even(source_bytes)
        L = self._hidden_dim
        num_tokens = (len(source_bytes) // 2) // L
        if num_tokens == 0:
            return struct.pack("<I", 0)
        dev = _staging.device()
        n_in = num_tokens * L * 2
        h_in = _staging.pinned(n_in, "in")
        _staging.fill_from(h_in, source_bytes)
        d_in = torch.empty(n_in, dtype=torch.uint8, device=dev)
        d_in.copy_(h_in, non_blocking=True)
        codes, scales = encode_rows(d_in.view(torch.bfloat16).view(num_tokens, L))
        n_sc = 2 * num_tokens
        h_out = _staging.pinned(n_sc + num_tokens * L, "out")
        h_out[:n_sc].copy_(scales.view(torch.uint8), non_blocking=True)
        h_out[n_sc:].copy_(codes.view(torch.uint8).view(-1), non_blocking=True)
        torch.cuda.current_stream(dev).synchronize()
        return _staging.to_bytes(h_out, struct.pack("<I", num_tokens))

    def decode(self, target_bytes: bytes) -> bytes:
        self._decode_calls += 1
        if len(target_bytes) < 4:
            return b""
        num_tokens = struct.unpack("<I", target_bytes[:4])[0]
        if num_tokens == 0:
            return b""
        L = self._hidden_dim
        n_sc, n_codes = 2 * num_tokens, num_tokens * L
        if len(target_bytes) < 4 + n_sc + n_codes:
            raise RuntimeError(f"INT8 blob too short: {len(target_bytes)} bytes for {num_tokens} tokens of "
                               f"{L} elements")
        dev = _staging.device()
        h_in = _staging.pinned(n_sc + n_codes, "in")
        _staging.fill_from(h_in, target_bytes, 4)
        d_sc = torch.empty(n_sc, dtype=torch.uint8, device=dev)
        d_codes = torch.empty(n_codes, dtype=torch.uint8, device=dev)
        d_sc.copy_(h_in[:n_sc], non_blocking=True)
        d_codes.copy_(h_in[n_sc:], non_blocking=True)
        out = decode_rows(d_codes.view(torch.int8).view(num_tokens, L), d_sc.view(torch.bfloat16))
        h_out = _staging.pinned(n_codes * 2, "out")
        h_out.copy_(out.view(torch.uint8).view(-1), non_blocking=True)
        torch.cuda.current_stream(dev).synchronize()
        return _staging.to_bytes(h_out)

    def checksum(self, raw_bytes: bytes) -> int:
        return checksum(raw_bytes)
