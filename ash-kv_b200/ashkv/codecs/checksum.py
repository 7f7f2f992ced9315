"""Checksums of page bytes.

``checksum``/``checksum_pair`` keep the reference's host semantics
(ashkv/codecs/checksum.py:26-55): XXH64 with seed 0 via the ``xxhash``
package when importable, else SHA-256 truncated to 8 little-endian bytes;
the pair adds MD5 truncated the same way.  These operate on host ``bytes``.

``checksum_pages`` computes the same XXH64 digest for many device-resident
pages in one sm_100a kernel launch (libashkv_cuda ``ashkv_xxh64_items``).
"""
from __future__ import annotations

import hashlib
from typing import Optional

import torch

try:
    import xxhash
    _HAS_XXHASH = True
except ImportError:  # pragma: no cover - xxhash is installed in the supported image
    _HAS_XXHASH = False


def _sha8(raw: bytes) -> int:
    return int.from_bytes(hashlib.sha256(raw).digest()[:8], "little", signed=False)


def checksum(raw_bytes: bytes) -> int:
    if _HAS_XXHASH:
        return xxhash.xxh64(raw_bytes).intdigest()
    return _sha8(raw_bytes)


def checksum_pair(raw_bytes: bytes) -> tuple[int, int]:
    a = checksum(raw_bytes)
    b = int.from_bytes(hashlib.md5(raw_bytes).digest()[:8], "little", signed=False)
    return a, b


def checksum_pages(pages: torch.Tensor, seed: int = 0, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """XXH64 of each row of a CUDA tensor [n_pages, ...] (row = one page's bytes).

    Returns an int64 CUDA tensor holding the digests' bit patterns
    (``.cpu().numpy().view(numpy.uint64)`` gives the unsigned values).
    """
    from .. import _native

    n = pages.shape[0]
    flat = pages.reshape(n, -1)
    if flat.stride(-1) != 1:
        raise ValueError("checksum_pages: pages must be row-contiguous")
    item_bytes = flat.shape[1] * flat.element_size()
    if out is None:
        out = torch.empty(n, dtype=torch.int64, device=pages.device)
    elif out.dtype != torch.int64 or out.numel() < n or not out.is_cuda:
        raise ValueError("checksum_pages: out must be an int64 CUDA tensor of at least n_pages entries")
    _native.xxh64_items(flat, n, item_bytes, flat.stride(0) * flat.element_size(), out, seed)
    return out
