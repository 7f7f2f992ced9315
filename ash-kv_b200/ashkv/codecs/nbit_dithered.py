"""Dithered N-bit (2/4/8) group codec with sigma-rule outlier isolation on sm_100a.

Drop-in for ``DitheredNBitCodec`` (ashkv/codecs/nbit_dithered.py:14-167 of
the reference): same constructor, same blob layout
``<II num_tokens, num_outliers> + bf16 delta[num_tokens*hidden_dim/32]
+ int32 outlier_index[] + bf16 outlier_value[] + packed codes`` (MSB-first),
same empty-input behaviour and the same SHA-256-based ``checksum``.

Dither.  The reference draws ``U = torch.rand(...)`` from a CUDA generator
seeded ``42 + encode_calls``.  Here ``encode`` generates the dither in-kernel
from Philox4x32-10 keyed by that same seed (a different random stream with
the same seeding policy: centred 8-bit uniforms U = (b + 0.5) / 256, 16 per
Philox draw, a dither resolution of 1/256 of the quantisation step).  Passing ``uniform=`` (the U tensor the
reference would draw) reproduces the reference's output bit for bit.

Device-resident entry points (no host copies): :func:`encode_groups`,
:func:`decode_groups` and :class:`NBitEncoded`.  Host-buffer entry points:
``encode_pinned`` / ``decode_pinned`` take and fill host tensors (pinned for
asynchronous DMA) holding the same blob as ``encode``/``decode``, with no
copy on the host.
"""
from __future__ import annotations

import hashlib
import math
import struct
from dataclasses import dataclass
from typing import Optional

import numpy as np
import torch

from .. import _native, _staging


def max_outliers_per_group(sigma: float, group: int = 32) -> int:
    """Bound on how many of ``group`` values can satisfy |x - mean| > sigma * std.

    With the unbiased std, m * sigma^2 < group - 1; one extra slot of margin
    absorbs rounding in the threshold.
    """
    if not sigma > 0:
        return group
    return int(min(group, math.floor((group - 1) / (sigma * sigma)) + 1))


@dataclass
class NBitEncoded:
    """Device-resident encoding of ``n_groups`` groups of 32 elements."""
    bits: int
    n_groups: int
    scales: torch.Tensor          # bf16 [n_groups]
    codes: torch.Tensor           # uint8 [n_groups * 32 * bits / 8]
    bucket_counts: torch.Tensor   # int32 [n_buckets] (true counts)
    bucket_entries: torch.Tensor  # int32 [n_buckets * bucket_cap]: (local_idx << 16) | bf16 bits
    bucket_cap: int
    status: torch.Tensor          # int32 [1], ASHKV_FLAG_* bits

    @property
    def n_buckets(self) -> int:
        return _native.nbit_bucket_count(self.n_groups)

    @staticmethod
    def allocate(n_groups: int, bits: int, bucket_cap: int, device: torch.device) -> "NBitEncoded":
        nb = _native.nbit_bucket_count(n_groups)
        return NBitEncoded(
            bits=bits, n_groups=n_groups,
            scales=torch.empty(n_groups, dtype=torch.bfloat16, device=device),
            codes=torch.empty(max(n_groups * 32 * bits // 8, 16), dtype=torch.uint8, device=device),
            bucket_counts=torch.empty(max(nb, 1), dtype=torch.int32, device=device),
            bucket_entries=torch.empty(max(nb * bucket_cap, 1), dtype=torch.int32, device=device),
            bucket_cap=bucket_cap,
            status=torch.zeros(1, dtype=torch.int32, device=device))


def encode_groups(src: torch.Tensor, bits: int, sigma: float = 3.0, *, uniform: Optional[torch.Tensor] = None,
                  seed: int = 42, dither_offset: int = 0, bucket_cap: Optional[int] = None,
                  out: Optional[NBitEncoded] = None) -> NBitEncoded:
    """Encode a contiguous bf16 CUDA tensor (numel a multiple of 32).

    ``bucket_cap`` defaults to the worst case for ``sigma`` (never overflows).
    ``out`` lets callers reuse preallocated buffers; its status word is
    cleared here.
    """
    n_groups = src.numel() // 32
    if out is None:
        if bucket_cap is None:
            bucket_cap = _native.NBIT_BUCKET_GROUPS * max_outliers_per_group(sigma)
        out = NBitEncoded.allocate(n_groups, bits, bucket_cap, src.device)
    else:
        out.status.zero_()
    _native.nbit_encode(src.reshape(-1), bits, sigma, out.scales, out.codes, out.bucket_counts,
                        out.bucket_entries, out.bucket_cap, out.status,
                        dither=None if uniform is None else uniform.reshape(-1), seed=seed,
                        dither_offset=dither_offset)
    return out


def decode_groups(enc: NBitEncoded, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Decode an :class:`NBitEncoded` back to bf16 (outliers restored)."""
    if out is None:
        out = torch.empty(enc.n_groups * 32, dtype=torch.bfloat16, device=enc.scales.device)
    _native.nbit_decode(enc.scales, enc.codes, enc.n_groups, enc.bits, out, enc.status,
                        enc.bucket_counts, enc.bucket_entries, enc.bucket_cap)
    return out


def flatten_outliers(enc: NBitEncoded) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Bucketed outliers -> (int32 flat index, bf16-bit values, total) on the device."""
    dev = enc.scales.device
    nb = enc.n_buckets
    cap_total = max(nb * enc.bucket_cap, 1)
    offsets = torch.empty(_native.nbit_flatten_scratch_ints(nb), dtype=torch.int32, device=dev)
    idx = torch.empty(cap_total, dtype=torch.int32, device=dev)
    val = torch.empty(cap_total, dtype=torch.int16, device=dev)
    total = torch.empty(1, dtype=torch.int32, device=dev)
    _native.nbit_outliers_flatten(enc.bucket_counts, enc.bucket_entries, enc.bucket_cap, nb, offsets, idx, val,
                                  total)
    return idx, val, total


def _host_flat(t: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """A contiguous host tensor viewed as a flat tensor of ``dtype`` (same bytes)."""
    if t.is_cuda:
        raise ValueError("expected a host tensor")
    if not t.is_contiguous():
        raise ValueError("host buffers must be contiguous")
    flat = t.reshape(-1)
    if flat.dtype != dtype:
        flat = flat.view(torch.uint8).view(dtype)
    return flat


def _host_out(out: Optional[torch.Tensor], n: int, dtype: torch.dtype) -> torch.Tensor:
    if out is None:
        return torch.empty(max(n, 1), dtype=dtype, pin_memory=torch.cuda.is_available())
    flat = _host_flat(out, dtype)
    if flat.numel() < n:
        raise ValueError(f"output buffer holds {flat.numel()} elements, {n} needed")
    return flat


def _host_bytes(data: bytes, out: Optional[torch.Tensor]) -> torch.Tensor:
    o = _host_out(out, len(data), torch.uint8)
    o[:len(data)].numpy()[:] = np.frombuffer(data, dtype=np.uint8)
    return o[:len(data)]


class PendingResult:
    """A queued host-buffer codec call; ``result()`` completes it (once) and returns its value.
    The buffers it writes must not be reused before ``result()`` returns."""

    __slots__ = ("_finish", "_value")

    def __init__(self, finish) -> None:
        self._finish = finish
        self._value = None

    def result(self):
        if self._finish is not None:
            self._value = self._finish()
            self._finish = None
        return self._value


_SIDE_STREAMS: dict = {}


def _side_streams(dev: torch.device, kind: str = "encode"):
    """Per-device (host->device, device->host) copy streams of the host-buffer API;
    encodes and decodes have their own pair, so the copies of one never queue
    behind the other's (the copy engines run both directions and both pairs at once)."""
    key = (dev.index, kind)
    if key not in _SIDE_STREAMS:
        _SIDE_STREAMS[key] = (torch.cuda.Stream(dev), torch.cuda.Stream(dev))
    return _SIDE_STREAMS[key]


# Host blob buffers whose device->host copies were queued without a host wait
# (encode_pinned_batch(host_sync=False)): data pointer -> CUDA event that
# completes with the copies.  decode_pinned_batch orders its reads of such a
# buffer after the event on the GPU; sync_host_blobs() waits on the host.
_BLOB_WRITES: dict = {}


def _record_blob_write(ptr: int, event) -> None:
    """Remember that the blob at host address ``ptr`` is complete once ``event`` is.
    Entries whose copies have already finished are dropped first, so blobs that are
    never decoded or synced do not accumulate (and a later buffer at a reused
    address never waits on a stale event)."""
    for k in [k for k, ev in _BLOB_WRITES.items() if ev.query()]:
        del _BLOB_WRITES[k]
    _BLOB_WRITES[ptr] = event


def sync_host_blobs(blobs) -> None:
    """Wait until the blobs returned by ``encode_pinned_batch(host_sync=False)`` are
    complete in host memory.  Needed before reading their bytes on the host (a
    blob passed to ``decode_pinned_batch`` is ordered on the GPU instead); a blob
    that is neither synced nor decoded is forgotten once its copies finish."""
    for b in blobs:
        ev = _BLOB_WRITES.pop(b.data_ptr(), None)
        if ev is not None:
            ev.synchronize()


def _sha8(raw: bytes) -> int:
    return int.from_bytes(hashlib.sha256(raw).digest()[:8], "little", signed=False)


class DitheredNBitCodec:
    """N-bit codec: group quantisation, sigma-rule outliers, stochastic dither."""

    __slots__ = ("_encode_calls", "_decode_calls", "_hidden_dim", "_group_size", "_sigma", "_bits",
                 "_num_states", "_half_states")

    def __init__(self, hidden_dim: int = 128, group_size: int = 32, sigma: float = 3.0, bits: int = 4) -> None:
        if bits not in (2, 4, 8):
            raise ValueError(f"DitheredNBitCodec only supports 2, 4, or 8 bits. Got: {bits}")
        if group_size != 32:
            raise ValueError(f"group_size must be 32 for the sm_100a kernel, got {group_size}")
        self._encode_calls = 0
        self._decode_calls = 0
        self._hidden_dim = hidden_dim
        self._group_size = group_size
        self._sigma = sigma
        self._bits = bits
        self._num_states = 2 ** bits
        self._half_states = (self._num_states - 1) / 2.0

    # The dither seed for this call (the reference seeds its generator the same way).
    def _seed(self) -> int:
        return 42 + self._encode_calls

    def checksum(self, raw_bytes: bytes) -> int:
        return _sha8(raw_bytes)

    def encode(self, source_bytes: bytes, *, uniform=None) -> bytes:
        """Encode bf16 bytes.  ``uniform`` (optional, fp32, one value per encoded
        element, CPU or CUDA) replaces the in-kernel dither with the given U."""
        self._encode_calls += 1
        if not source_bytes:
            return struct.pack("<II", 0, 0)
        _staging.check_even(source_bytes)
        L = self._hidden_dim
        num_tokens = (len(source_bytes) // 2) // L
        if num_tokens == 0:
            return struct.pack("<II", 0, 0)
        if L % self._group_size:
            raise RuntimeError(f"shape '[{num_tokens}, {L // self._group_size}, {self._group_size}]' is invalid "
                               f"for input of size {num_tokens * L}")
        dev = _staging.device()
        n_elems = num_tokens * L
        h_in = _staging.pinned(2 * n_elems, "in")
        _staging.fill_from(h_in, source_bytes)
        d_src = torch.empty(2 * n_elems, dtype=torch.uint8, device=dev)
        d_src.copy_(h_in, non_blocking=True)
        u = None
        if uniform is not None:
            u = torch.as_tensor(uniform, dtype=torch.float32).reshape(-1)
            if u.numel() != n_elems:
                raise ValueError(f"uniform has {u.numel()} values, expected {n_elems}")
            u = u.to(dev, non_blocking=True).contiguous()
        enc = encode_groups(d_src.view(torch.bfloat16), self._bits, self._sigma, uniform=u, seed=self._seed())
        idx, val, total = flatten_outliers(enc)
        n_out = int(total.item())  # one sync: the blob layout depends on the outlier count
        n_groups = enc.n_groups
        n_codes = n_groups * 32 * self._bits // 8
        size = 2 * n_groups + 6 * n_out + n_codes
        h_out = _staging.pinned(size, "out")
        o = 0
        h_out[o:o + 2 * n_groups].copy_(enc.scales.view(torch.uint8), non_blocking=True); o += 2 * n_groups
        if n_out:
            h_out[o:o + 4 * n_out].copy_(idx[:n_out].view(torch.uint8), non_blocking=True); o += 4 * n_out
            h_out[o:o + 2 * n_out].copy_(val[:n_out].view(torch.uint8), non_blocking=True); o += 2 * n_out
        h_out[o:o + n_codes].copy_(enc.codes[:n_codes], non_blocking=True)
        torch.cuda.current_stream(dev).synchronize()
        return _staging.to_bytes(h_out, struct.pack("<II", num_tokens, n_out))

    # ---------------------------------------------------------------- host tensors
    def encode_pinned(self, src: torch.Tensor, out: Optional[torch.Tensor] = None, *, uniform=None) -> torch.Tensor:
        """Encode a contiguous host tensor of bf16 values into the blob ``encode``
        returns for the same bytes, written into the host uint8 tensor ``out``
        (allocated pinned when None); returns ``out[:blob_size]``.

        With pinned buffers the host<->device transfers are DMA copies straight
        from ``src`` and into ``out``; the call returns once ``out`` is complete."""
        return self.encode_pinned_batch([src], [out], uniforms=[uniform])[0]

    def encode_pinned_batch(self, srcs, outs=None, *, uniforms=None, wait: bool = True,
                            host_sync: bool = True):
        """``encode_pinned`` over several tensors, in order (one call each, so each
        gets the seed that call would get).  Host->device copies run on one side
        stream and device->host copies on another, so a tensor's blob travels
        back while the next tensor's input is still arriving.

        With ``wait=False`` the call returns a :class:`PendingResult` once the
        copies in and the kernels are queued; ``.result()`` then reads the outlier
        counts, queues the copies out and returns the list of blobs.  Work queued
        in between (for example the decode of the previous blobs) overlaps it.

        With ``host_sync=False`` the blobs are returned as soon as their copies out
        are queued: their 8-byte headers are final, the rest lands when the copies
        complete.  ``decode_pinned_batch`` may be given such blobs directly (it
        orders its reads after the copies on the GPU); ``sync_host_blobs(blobs)``
        waits for them before the host reads their bytes.  The output buffers must
        not be handed to another encode until the blobs' decode has completed."""
        outs = list(outs) if outs is not None else [None] * len(srcs)
        uniforms = list(uniforms) if uniforms is not None else [None] * len(srcs)
        if not (len(outs) == len(uniforms) == len(srcs)):
            raise ValueError("srcs, outs and uniforms must have the same length")
        L = self._hidden_dim
        dev = None
        totals = None
        jobs = []
        for src in srcs:
            flat = _host_flat(src, torch.bfloat16)
            num_tokens = flat.numel() // L
            if num_tokens and L % self._group_size:
                raise RuntimeError(f"shape '[{num_tokens}, {L // self._group_size}, {self._group_size}]' is invalid "
                                   f"for input of size {num_tokens * L}")
            jobs.append({"flat": flat, "num_tokens": num_tokens})
        if any(j["num_tokens"] for j in jobs):
            dev = _staging.device()
            cur = torch.cuda.current_stream(dev)
            h2d, d2h = _side_streams(dev)
            h2d.wait_stream(cur)   # device buffers below may reuse memory the current stream still uses
            for j, u in zip(jobs, uniforms):
                if not j["num_tokens"]:
                    continue
                n_elems = j["num_tokens"] * L
                j["d_src"] = torch.empty(n_elems, dtype=torch.bfloat16, device=dev)
                if u is not None:
                    u = torch.as_tensor(u, dtype=torch.float32).reshape(-1)
                    if u.numel() != n_elems:
                        raise ValueError(f"uniform has {u.numel()} values, expected {n_elems}")
                with torch.cuda.stream(h2d):
                    j["d_src"].copy_(j["flat"][:n_elems], non_blocking=True)
                    j["u"] = None if u is None else u.to(dev, non_blocking=True).contiguous()
                # the buffers come from the current stream's pool but are written on h2d:
                # tell the caching allocator, so a free cannot hand them out while h2d is busy
                j["d_src"].record_stream(h2d)
                if j["u"] is not None:
                    j["u"].record_stream(h2d)
                j["ready"] = h2d.record_event()
            totals = torch.empty(len(jobs), dtype=torch.int32, pin_memory=True)
        for i, j in enumerate(jobs):
            self._encode_calls += 1
            if not j["num_tokens"]:
                continue
            cur.wait_event(j["ready"])
            enc = encode_groups(j["d_src"], self._bits, self._sigma, uniform=j["u"], seed=self._seed())
            idx, val, total = flatten_outliers(enc)
            totals[i:i + 1].copy_(total, non_blocking=True)
            j.update(enc=enc, idx=idx, val=val, done=cur.record_event())

        def finish():
            return self._encode_finish(jobs, outs, totals, dev, host_sync)
        return finish() if wait else PendingResult(finish)

    def _encode_finish(self, jobs, outs, totals, dev, host_sync: bool = True) -> list:
        d2h = _side_streams(dev)[1] if dev is not None else None
        results = []
        for i, (j, out) in enumerate(zip(jobs, outs)):
            if not j["num_tokens"]:
                results.append(_host_bytes(struct.pack("<II", 0, 0), out))
                continue
            j["done"].synchronize()
            n_out = int(totals[i])
            enc = j["enc"]
            n_groups = enc.n_groups
            n_codes = n_groups * 32 * self._bits // 8
            size = 8 + 2 * n_groups + 6 * n_out + n_codes
            out = _host_out(out, size, torch.uint8)
            out[:8].numpy()[:] = np.frombuffer(struct.pack("<II", j["num_tokens"], n_out), dtype=np.uint8)
            d2h.wait_event(j["done"])
            with torch.cuda.stream(d2h):
                o = 8
                out[o:o + 2 * n_groups].copy_(enc.scales.view(torch.uint8), non_blocking=True); o += 2 * n_groups
                if n_out:
                    out[o:o + 4 * n_out].copy_(j["idx"][:n_out].view(torch.uint8), non_blocking=True); o += 4 * n_out
                    out[o:o + 2 * n_out].copy_(j["val"][:n_out].view(torch.uint8), non_blocking=True); o += 2 * n_out
                out[o:o + n_codes].copy_(enc.codes[:n_codes], non_blocking=True)
            # read on d2h, possibly after this call returns (host_sync=False)
            for t in (enc.scales, enc.codes, j["idx"], j["val"]):
                t.record_stream(d2h)
            results.append(out[:size])
        if dev is not None:
            copied = d2h.record_event()
            if host_sync:
                copied.synchronize()
            else:
                for r in results:
                    if r.numel() > 8:
                        _record_blob_write(r.data_ptr(), copied)
        return results

    def decode_pinned(self, blob: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Decode a blob held in a host uint8 tensor into the host bf16 tensor
        ``out`` (allocated pinned when None); returns ``out[:n]``, the values
        ``decode`` returns for the same bytes."""
        return self.decode_pinned_batch([blob], [out])[0]

    def decode_pinned_batch(self, blobs, outs=None, *, wait: bool = True):
        """``decode_pinned`` over several blobs; a blob's values travel back to the
        host while the next blob is still being copied in and decoded.  With
        ``wait=False`` returns a :class:`PendingResult` once everything is queued."""
        outs = list(outs) if outs is not None else [None] * len(blobs)
        if len(outs) != len(blobs):
            raise ValueError("blobs and outs must have the same length")
        jobs = []
        for blob in blobs:
            self._decode_calls += 1
            b = _host_flat(blob, torch.uint8)
            num_tokens = n_out = 0
            if b.numel() >= 8:
                num_tokens, n_out = struct.unpack("<II", b[:8].numpy().tobytes())
            j = {"b": b, "num_tokens": num_tokens, "n_out": n_out}
            if num_tokens:
                n_groups = num_tokens * (self._hidden_dim // self._group_size)
                n_codes = n_groups * 32 * self._bits // 8
                need = 8 + 2 * n_groups + 6 * n_out + n_codes
                if b.numel() < need:
                    raise RuntimeError(f"N-bit blob too short: {b.numel()} bytes, layout needs {need}")
                j.update(n_groups=n_groups, n_codes=n_codes)
            jobs.append(j)
        dev = None
        if any(j["num_tokens"] for j in jobs):
            dev = _staging.device()
            cur = torch.cuda.current_stream(dev)
            h2d, d2h = _side_streams(dev, "decode")
            h2d.wait_stream(cur)
            for j in jobs:
                if not j["num_tokens"]:
                    continue
                b, g, nc, n_out = j["b"], j["n_groups"], j["n_codes"], j["n_out"]
                written = _BLOB_WRITES.pop(b.data_ptr(), None)
                if written is not None:  # blob bytes still arriving from an encode
                    h2d.wait_event(written)
                # one DMA per blob section, each into its own (aligned) device buffer
                d_sc = torch.empty(2 * g, dtype=torch.uint8, device=dev)
                d_idx = torch.empty(max(4 * n_out, 4), dtype=torch.uint8, device=dev)
                d_val = torch.empty(max(2 * n_out, 2), dtype=torch.uint8, device=dev)
                codes = torch.empty(max(nc, 16), dtype=torch.uint8, device=dev)
                with torch.cuda.stream(h2d):
                    o = 8
                    d_sc.copy_(b[o:o + 2 * g], non_blocking=True); o += 2 * g
                    if n_out:
                        d_idx[:4 * n_out].copy_(b[o:o + 4 * n_out], non_blocking=True); o += 4 * n_out
                        d_val[:2 * n_out].copy_(b[o:o + 2 * n_out], non_blocking=True); o += 2 * n_out
                    codes[:nc].copy_(b[o:o + nc], non_blocking=True)
                for t in (d_sc, d_idx, d_val, codes):  # written on h2d (see encode_pinned_batch)
                    t.record_stream(h2d)
                j.update(d_sc=d_sc, d_idx=d_idx, d_val=d_val, codes=codes, ready=h2d.record_event())
            statuses = torch.zeros(len(jobs), dtype=torch.int32, device=dev)
            h_status = torch.empty(len(jobs), dtype=torch.int32, pin_memory=True)
        results = []
        for i, (j, out) in enumerate(zip(jobs, outs)):
            if not j["num_tokens"]:
                results.append(_host_out(out, 0, torch.bfloat16)[:0])
                continue
            g, n_out = j["n_groups"], j["n_out"]
            cur.wait_event(j["ready"])
            dv = torch.empty(g * 32, dtype=torch.bfloat16, device=dev)
            _native.nbit_decode_flat(j["d_sc"].view(torch.bfloat16), j["codes"], g, self._bits,
                                     j["d_idx"].view(torch.int32) if n_out else None,
                                     j["d_val"].view(torch.int16) if n_out else None, n_out, dv,
                                     statuses[i:i + 1])
            done = cur.record_event()
            out = _host_out(out, g * 32, torch.bfloat16)
            d2h.wait_event(done)
            with torch.cuda.stream(d2h):
                out[:g * 32].copy_(dv, non_blocking=True)
            dv.record_stream(d2h)
            j["dv"] = dv
            results.append(out[:g * 32])
        done = None
        if dev is not None:
            d2h.wait_stream(cur)
            with torch.cuda.stream(d2h):
                h_status.copy_(statuses, non_blocking=True)
            statuses.record_stream(d2h)  # read on d2h after this call returns (wait=False)
            done = d2h.record_event()

        def finish():
            if done is not None:
                done.synchronize()
                for i, j in enumerate(jobs):
                    if j["num_tokens"] and int(h_status[i]) & _native.FLAG_INDEX_RANGE:
                        raise IndexError(f"outlier index out of range for a decoded size of "
                                         f"{j['n_groups'] * 32} elements")
            return results
        return finish() if wait else PendingResult(finish)

    def decode(self, target_bytes: bytes) -> bytes:
        self._decode_calls += 1
        if len(target_bytes) < 8:
            return b""
        num_tokens, n_out = struct.unpack("<II", target_bytes[:8])
        if num_tokens == 0:
            return b""
        groups_per_row = self._hidden_dim // self._group_size
        n_groups = num_tokens * groups_per_row
        n_codes = n_groups * 32 * self._bits // 8
        need = 8 + 2 * n_groups + 6 * n_out + n_codes
        if len(target_bytes) < need:
            raise RuntimeError(f"N-bit blob too short: {len(target_bytes)} bytes, layout needs {need}")
        dev = _staging.device()
        body = len(target_bytes) - 8
        h_in = _staging.pinned(body, "in")
        _staging.fill_from(h_in, target_bytes, 8)
        d_sc = torch.empty(2 * n_groups, dtype=torch.uint8, device=dev)
        d_idx = torch.empty(max(4 * n_out, 4), dtype=torch.uint8, device=dev)
        d_val = torch.empty(max(2 * n_out, 2), dtype=torch.uint8, device=dev)
        d_codes = torch.empty(max(n_codes, 16), dtype=torch.uint8, device=dev)
        o = 0
        d_sc.copy_(h_in[o:o + 2 * n_groups], non_blocking=True); o += 2 * n_groups
        if n_out:
            d_idx[:4 * n_out].copy_(h_in[o:o + 4 * n_out], non_blocking=True); o += 4 * n_out
            d_val[:2 * n_out].copy_(h_in[o:o + 2 * n_out], non_blocking=True); o += 2 * n_out
        d_codes[:n_codes].copy_(h_in[o:o + n_codes], non_blocking=True)
        out = torch.empty(n_groups * 32, dtype=torch.bfloat16, device=dev)
        status = torch.zeros(1, dtype=torch.int32, device=dev)
        _native.nbit_decode_flat(d_sc.view(torch.bfloat16), d_codes, n_groups, self._bits,
                                 d_idx.view(torch.int32) if n_out else None,
                                 d_val.view(torch.int16) if n_out else None, n_out, out, status)
        h_out = _staging.pinned(2 * n_groups * 32, "out")
        h_out.copy_(out.view(torch.uint8), non_blocking=True)
        st = status.to("cpu", non_blocking=True)
        torch.cuda.current_stream(dev).synchronize()
        if int(st.item()) & _native.FLAG_INDEX_RANGE:
            raise IndexError(f"outlier index out of range for a decoded size of {n_groups * 32} elements")
        return _staging.to_bytes(h_out)
