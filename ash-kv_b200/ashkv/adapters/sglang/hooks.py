"""SGLang HiCache IO interception on sm_100a.

Drop-in for ``SGLangHooks`` (ashkv/adapters/sglang/hooks.py:20-245 of the
reference).  Same constructor, ``stats`` keys, debounced JSON stats file,
``compressible_layers`` semantics, return values (``False`` declines and
lets SGLang run its native copy) and host-slot byte format:

    slot(token t, layer l) = 2 * head_num * head_dim bytes:
      [0, 2H)            fp16 scales of tokens t*H .. t*H+H-1 (see below)
      [2H, 2H + H*D)     int8 codes of token t (one absmax scale per token
                         over all local heads)
      [2H + H*D, 2*H*D)  zero

The reference writes token t's scale at flat index t of a [num_tokens, H]
buffer and then copies that buffer to the slots H entries at a time, so slot
t carries the scales of tokens t*H .. t*H+H-1; promote reads them back the
same way.  This module keeps that placement byte for byte (entries past the
last token, which the reference leaves uninitialised, are zero here).

Differences in how the work is done:
  * demote: one gather+encode launch over all layers for K and one for V
    writes the packed slots straight into a reused device staging buffer
    [tokens, layers, slot]; a single pitched device->host copy each moves all
    layers, and the hook waits once for both (the reference runs one Triton
    launch, two synchronous .cpu() copies and a host scatter per layer).  With
    ``compact_host_slots`` (the default) that copy carries only the used
    2H + H*D bytes of each compressed slot, so the bytes saved are saved on
    the link too; the zero tail [2H + H*D, 2*H*D), which nothing reads, is
    then left as it was in the host pool.  ``compact_host_slots = False``
    writes whole slots, zero tail included, byte for byte as the reference;
  * promote: a pitched host->device copy moves only the used 2H + H*D bytes
    of each slot, and the decode kernel scatters rows straight into the
    device pool at ``device_indices``;
  * layers outside ``compressible_layers`` are copied as bf16 in both
    directions (the reference's ``tensor[index].copy_()`` there writes into
    a temporary produced by advanced indexing, so those copies never land).
"""
from __future__ import annotations

import json
import logging
import os
import time
from typing import Any

import numpy as np
import torch

from ... import _native
from ...safety.circuit_breaker import CircuitBreakerRegistry

logger = logging.getLogger("ashkv.adapters.sglang.hooks")


def _contiguous_range(idx: torch.Tensor) -> int | None:
    """First index if ``idx`` is an ascending run of consecutive integers, else None."""
    n = idx.numel()
    if n == 0:
        return None
    a = idx.detach().to("cpu", torch.int64).reshape(-1).numpy()  # host indices: no copy
    first = int(a[0])
    if n == 1 or (int(a[-1]) - first == n - 1 and bool((np.diff(a) == 1).all())):
        return first
    return None


def _ceil16(n: int) -> int:
    return (n + 15) // 16 * 16


class SGLangHooks:
    """Demote (GPU -> CPU, compress) and promote (CPU -> GPU, decompress) hooks."""

    def __init__(self, codec_name: str = "int8_default"):
        self.codec_name = codec_name
        self.circuit_breaker = CircuitBreakerRegistry()
        self.compressible_layers = None
        self.compact_host_slots = True
        self.transfer_stats = {"d2h_bytes": 0, "h2d_bytes": 0}  # bytes moved over the host link
        self._stage_bufs: dict = {}  # device -> reusable staging buffer
        self._ptr_cache: dict = {}   # (device, layer addresses) -> device table of them
        self.stats = {"tokens_compressed": 0, "tokens_decompressed": 0, "bytes_saved": 0,
                      "blocks_intercepted": 0, "last_flush_time": 0}
        os.makedirs("stats", exist_ok=True)
        self.stats_file = "stats/ashkv_stats.json"
        self._flush_stats()

    # ------------------------------------------------------------------ stats
    def _flush_stats(self) -> None:
        try:
            with open(self.stats_file, "w") as f:
                json.dump(self.stats, f)
        except Exception as e:  # never let telemetry break the IO path
            logger.warning("[ASH-KV] Failed to flush stats: %s", e)

    def _maybe_flush(self) -> None:
        if time.time() - self.stats["last_flush_time"] > 1.0:
            self._flush_stats()
            self.stats["last_flush_time"] = time.time()

    # ------------------------------------------------------------------ demote
    def demote_hook(self, device_pool: Any, host_pool: Any, host_indices: torch.Tensor,
                    device_indices: torch.Tensor, pool_type: str, io_backend: Any = None) -> bool:
        if pool_type != "MHA":
            return False
        n = len(device_indices)
        if n == 0:
            return False
        H, D, L = device_pool.head_num, device_pool.head_dim, device_pool.layer_num
        if self.compressible_layers is None:
            self.compressible_layers = list(range(L))
        self._demote(device_pool, host_pool, host_indices, device_indices, n, H, D, L,
                     set(self.compressible_layers))
        row = H * D
        nc = len(self.compressible_layers)
        self.stats["blocks_intercepted"] += 1
        self.stats["tokens_compressed"] += n * nc
        bf16_bytes = n * nc * row * 2 * 2
        int8_bytes = n * nc * (row + 2 * H) * 2
        self.stats["bytes_saved"] += bf16_bytes - int8_bytes
        self._maybe_flush()
        return True

    def _demote(self, device_pool, host_pool, host_indices, device_indices, n, H, D, L, compress) -> None:
        dev = device_pool.k_buffer[0].device
        if dev.type != "cuda":
            raise RuntimeError("SGLangHooks needs the device KV pool on a CUDA device")
        with torch.cuda.device(dev):
            self._demote_cuda(device_pool, host_pool, host_indices, device_indices, n, H, D, L, compress)

    def _staging(self, dev: torch.device, nbytes: int) -> torch.Tensor:
        """A device byte buffer reused across calls (grown when a call needs more)."""
        buf = self._stage_bufs.get(dev)
        if buf is None or buf.numel() < nbytes:
            buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=dev)
            self._stage_bufs[dev] = buf
        return buf[:nbytes]

    def _layer_ptrs(self, layers, dev: torch.device) -> torch.Tensor:
        key = (dev, tuple(t.data_ptr() for t in layers))
        t = self._ptr_cache.get(key)
        if t is None:
            if len(self._ptr_cache) > 16:
                self._ptr_cache.clear()
            t = torch.tensor(list(key[1]), dtype=torch.int64, device=dev)
            self._ptr_cache[key] = t
        return t

    def _demote_cuda(self, device_pool, host_pool, host_indices, device_indices, n, H, D, L, compress) -> None:
        row, slot = H * D, 2 * H * D
        dev = device_pool.k_buffer[0].device
        didx = device_indices.to(device=dev, dtype=torch.int64)
        # staging [K/V, token, layer, slot]: the host pools' row order, so each of K and V
        # leaves in one pitched copy
        staging = self._staging(dev, 2 * n * L * slot).view(2, n, L, slot)
        # scale entries past the last token stay zero; with whole slots the zero tail travels too
        staging[:, :, :, :2 * H].zero_()
        if not self.compact_host_slots:
            staging[:, :, :, 2 * H + row:].zero_()
        elif (2 * H + row) % 16:  # an indexed host scatter moves whole 16-byte chunks: pad with zeros
            staging[:, :, :, 2 * H + row:_ceil16(2 * H + row)].zero_()
        all_layers = len(compress) == L
        pinned = False
        for kv, name in enumerate(("k_buffer", "v_buffer")):
            dbuf = getattr(device_pool, name)
            st = staging[kv]
            layers = [dbuf[layer] for layer in range(L)]
            if all_layers and all(t.is_contiguous() and t.data_ptr() % 16 == 0 for t in layers):
                # one launch over every layer: layer l's codes at slot l of each token row
                _native.int8_encode_rows_layers(
                    self._layer_ptrs(layers, dev), L, layers[0].dtype, row, row, didx, n,
                    st.data_ptr() + 2 * H, L * slot, slot, st.data_ptr(), H, L * slot, slot, dev)
            else:
                flat = st.reshape(-1)
                for layer in range(L):
                    src = layers[layer].view(-1, row)
                    if layer in compress:
                        codes = st[:, layer, 2 * H:2 * H + row].view(torch.int8)
                        # scale of token t -> st[t // H, layer, 2 * (t % H)]
                        scales = flat[layer * slot:].view(torch.float16)
                        _native.int8_encode_rows(src, codes, scales, row_index=didx, scales_per_slot=H,
                                                 scale_slot_stride=L * slot)
                    else:
                        st[:, layer, :].view(torch.bfloat16).copy_(src[didx].view(n, row))
            widths = [2 * H + row if (self.compact_host_slots and layer in compress) else slot for layer in range(L)]
            hbuf = getattr(host_pool, name)
            self._write_host_rows(hbuf, host_indices, st, n, L, slot, widths)
            pinned |= hbuf.is_pinned()
            self.transfer_stats["d2h_bytes"] += n * sum(widths)
        if pinned:  # the host pool is complete when the hook returns, as after the reference's .cpu() copies
            torch.cuda.current_stream(dev).synchronize()

    @staticmethod
    def _write_host_rows(host_buf: torch.Tensor, host_indices, staging: torch.Tensor, n: int, L: int,
                         slot: int, widths: list[int]) -> None:
        """Copy the first widths[l] bytes of each staging slot [n, L, slot] into host rows
        host_buf[host_indices] (each row [L, H, D] bf16, i.e. L slots of `slot` bytes)."""
        hview = host_buf.view(host_buf.shape[0], -1).view(torch.uint8)
        first = _contiguous_range(host_indices) if host_buf.is_contiguous() else None
        if first is not None:
            dst = hview[first:first + n]
            if all(w == slot for w in widths):
                dst.copy_(staging.view(n, L * slot), non_blocking=host_buf.is_pinned())
            elif len(set(widths)) == 1:  # one pitched copy over all (token, layer) slots
                _native.memcpy2d(dst.data_ptr(), slot, staging.data_ptr(), slot, widths[0], n * L, staging.device)
            else:
                for layer, w in enumerate(widths):
                    _native.memcpy2d(dst.data_ptr() + layer * slot, L * slot, staging.data_ptr() + layer * slot,
                                     L * slot, w, n, staging.device)
        elif host_buf.is_pinned() and host_buf.is_contiguous():
            # scattered rows: one kernel writes the slots into the pinned pool through its device mapping
            hidx = host_indices.detach().to(staging.device, torch.int64)
            groups = [(0, L, widths[0])] if len(set(widths)) == 1 else [(layer, 1, w) for layer, w in enumerate(widths)]
            for first_layer, n_sub, w in groups:
                _native.copy_rows_indexed(host_buf.data_ptr() + first_layer * slot, L * slot, slot, hidx,
                                          host_buf.shape[0], staging.data_ptr() + first_layer * slot, L * slot,
                                          slot, None, n, _ceil16(w), n_sub, n, staging.device)
        else:
            hidx = host_indices.detach().to("cpu", torch.int64)
            h3 = hview.view(hview.shape[0], L, slot)
            if all(w == slot for w in widths):
                hview[hidx] = staging.view(n, L * slot).to("cpu")
            elif len(set(widths)) == 1:
                w = widths[0]
                h3[hidx, :, :w] = staging[:, :, :w].contiguous().to("cpu")
            else:
                bounce = staging.to("cpu")
                for layer, w in enumerate(widths):
                    h3[hidx, layer, :w] = bounce[:, layer, :w]

    # ------------------------------------------------------------------ promote
    def promote_hook(self, device_pool: Any, host_pool: Any, host_indices: torch.Tensor,
                     device_indices: torch.Tensor, layer_id: int, pool_type: str, io_backend: Any = None) -> bool:
        if pool_type != "MHA":
            return False
        n = len(device_indices)
        if n == 0:
            return False
        H, D = device_pool.head_num, device_pool.head_dim
        dev = device_pool.k_buffer[0].device
        if dev.type != "cuda":
            raise RuntimeError("SGLangHooks needs the device KV pool on a CUDA device")
        native_layer = self.compressible_layers is not None and layer_id not in self.compressible_layers
        with torch.cuda.device(dev):
            self._promote_cuda(device_pool, host_pool, host_indices, device_indices, layer_id, H, D, native_layer)
        if not native_layer:
            self.stats["tokens_decompressed"] += n
            self._maybe_flush()
        return True

    def _promote_cuda(self, device_pool, host_pool, host_indices, device_indices, layer_id, H, D,
                      native_layer: bool) -> None:
        row, slot = H * D, 2 * H * D
        n = len(device_indices)
        dev = device_pool.k_buffer[0].device
        didx = device_indices.to(device=dev, dtype=torch.int64)
        used = slot if native_layer else 2 * H + row
        self.transfer_stats["h2d_bytes"] += 2 * n * used
        first = _contiguous_range(host_indices)  # once for K and V (SGLang calls this hook per layer)
        hidx = {}
        for name in ("k_buffer", "v_buffer"):
            hbuf = getattr(host_pool, name)
            L = hbuf.shape[1]
            upad = _ceil16(used)  # staged rows padded to 16 bytes for the indexed gather
            staged = torch.empty((n, upad), dtype=torch.uint8, device=dev)
            self._read_host_slots(hbuf, host_indices, layer_id, staged, n, L, slot, used, first, hidx)
            dst = getattr(device_pool, name)[layer_id].view(-1, row)
            if native_layer:
                dst[didx] = staged.view(torch.bfloat16).view(n, row)
                continue
            codes = staged[:, 2 * H:2 * H + row].view(torch.int8)
            scales = staged.view(-1).view(torch.float16)
            _native.int8_decode_rows(codes, scales, dst, row_index=didx, scales_per_slot=H,
                                     scale_slot_stride=upad)

    @staticmethod
    def _read_host_slots(hbuf: torch.Tensor, host_indices, layer_id: int, staged: torch.Tensor, n: int, L: int,
                         slot: int, used: int, first: int | None, hidx: dict) -> None:
        """``first``: the contiguity of ``host_indices`` (from _contiguous_range); ``hidx`` caches
        the indices' device copy between the K and V calls."""
        first = first if hbuf.is_contiguous() else None
        upad = staged.shape[1]
        if first is not None:
            base = hbuf.data_ptr() + (first * L + layer_id) * slot
            _native.memcpy2d(staged.data_ptr(), upad, base, L * slot, used, n, staged.device)
            if not hbuf.is_pinned():
                torch.cuda.current_stream(staged.device).synchronize()
        elif hbuf.is_pinned() and hbuf.is_contiguous():
            # scattered rows: one kernel reads the slots from the pinned pool through its device mapping
            if "dev" not in hidx:
                hidx["dev"] = host_indices.detach().to(staged.device, torch.int64)
            _native.copy_rows_indexed(staged.data_ptr(), upad, 0, None, n, hbuf.data_ptr() + layer_id * slot,
                                      L * slot, 0, hidx["dev"], hbuf.shape[0], upad, 1, n, staged.device)
        else:
            hidx = host_indices.detach().to("cpu", torch.int64)
            rows = hbuf[hidx, layer_id].contiguous().view(n, -1).view(torch.uint8)[:, :used]
            staged[:, :used].copy_(rows)
