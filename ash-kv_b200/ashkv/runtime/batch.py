"""Batched, device-resident page migration (the per-step hot path).

The reference applies ``score_vectorized`` -> ``desired_tiers`` to a host
snapshot of the page table and would call ``migrate`` once per page
(ashkv/runtime/migrate.py:35-191), moving bytes through the host for every
page.  Here one decode step is a handful of kernel launches with no host round
trip:

1. ``ashkv_policy_step``    score -> desired tier -> stable demote / promote lists
2. ``ashkv_migrate_pages``  every listed page, whatever its (current, target)
                            tier edge, is decoded from its current tier's store
                            and encoded into a slot of the target tier's store
                            (or back into its KV-pool rows); tier and slot are
                            committed in the device page table
3. ``ashkv_release_slots``  the slots pages gave up go back on their stores'
                            free stacks

List lengths stay on the device; every kernel reads them there.  Each tier
has its own :class:`TierStore` whose page format follows the codec the
resolver puts on the edge into that tier (``ashkv.compiler.tier_formats``):
BF16 pages live in the KV pool, the FP8 tier holds INT8 (the hooks' per-token
layout) or FP8 pages, the INT4 tier INT4Codec or dithered 4-bit pages, the
archive tier dithered INT2 pages.

As in ``migrate()``, pinned pages, pages already at their target and tiers
without a codec are skipped and reported per entry; a slot is taken only for
a page that moves, and the slot a page leaves is released in the same step.

``Int8PageCodec`` keeps the raw BF16 <-> INT8 page kernels
(``ashkv_int8_encode_pages`` / ``_decode_pages``) for callers that manage
tiers themselves.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Mapping, Optional, Sequence

import numpy as np
import torch

from .. import _native
from ..compiler.runtime_builder import controller_tables
from ..contracts.config import ASHKVConfig
from ..contracts.page import PageTable
from ..contracts.tiers import Tier

NUM_TIERS = 6


@dataclass
class DevicePageTable:
    """GPU mirror (struct of arrays) of the PageTable columns the hot path reads."""
    T: torch.Tensor
    S: torch.Tensor
    N: torch.Tensor
    P: torch.Tensor
    tier: torch.Tensor         # int8
    pin: torch.Tensor          # int32
    layer: torch.Tensor        # int32
    token_start: torch.Tensor  # int32
    slot: torch.Tensor         # int32, slot of the page in its tier's store, or -1

    @property
    def n(self) -> int:
        return self.T.numel()

    @staticmethod
    def empty(n: int, device: torch.device) -> "DevicePageTable":
        f = lambda dt: torch.zeros(n, dtype=dt, device=device)  # noqa: E731
        t = DevicePageTable(f(torch.float32), f(torch.float32), f(torch.float32), f(torch.float32),
                            f(torch.int8), f(torch.int32), f(torch.int32), f(torch.int32), f(torch.int32))
        t.slot.fill_(-1)
        return t

    @staticmethod
    def from_host(table: PageTable, device: torch.device) -> "DevicePageTable":
        cols = table.columns()
        up = lambda name, dt: torch.from_numpy(np.ascontiguousarray(cols[name]).astype(dt)).to(device)  # noqa: E731
        slot = torch.full((len(cols),), -1, dtype=torch.int32, device=device)
        return DevicePageTable(up("T", np.float32), up("S", np.float32), up("N", np.float32), up("P", np.float32),
                               up("tier", np.int8), up("pin_count", np.int32), up("layer_id", np.int32),
                               up("token_start", np.int32), slot)

    def update_scores(self, table: PageTable) -> None:
        cols = table.columns()
        for name in ("T", "S", "N", "P"):
            getattr(self, name).copy_(torch.from_numpy(np.ascontiguousarray(cols[name])), non_blocking=False)


class SlotArena:
    """Fixed-size slots in one device buffer with a device-side free stack."""

    def __init__(self, n_slots: int, slot_bytes: int, device: torch.device):
        if slot_bytes % 16:
            raise ValueError("slot_bytes must be a multiple of 16")
        self.n_slots, self.slot_bytes = n_slots, slot_bytes
        self.data = torch.empty(max(n_slots, 1) * slot_bytes, dtype=torch.uint8, device=device)
        # slot 0 on top of the stack first
        self.free_stack = torch.arange(n_slots - 1, -1, -1, dtype=torch.int32, device=device)
        self.free_top = torch.full((1,), n_slots, dtype=torch.int32, device=device)

    def free_count(self) -> int:
        return int(self.free_top.item())

    def pressure(self) -> float:
        return 1.0 - self.free_count() / max(self.n_slots, 1)

    def pressure_tensor(self) -> torch.Tensor:
        """Occupied fraction as a one-element float32 device tensor (no host sync)."""
        return 1.0 - self.free_top.float() / float(max(self.n_slots, 1))

    def slot_view(self) -> torch.Tensor:
        return self.data[: self.n_slots * self.slot_bytes].view(self.n_slots, self.slot_bytes)


class TierStore(SlotArena):
    """The slots of one tier: ``n_slots`` pages in ``fmt`` (an ``_native.PAGE_*`` format)."""

    def __init__(self, fmt: int, n_slots: int, device: torch.device, tokens_per_page: int, row_len: int,
                 outlier_cap: int = 0):
        need = _native.page_slot_bytes(fmt, tokens_per_page, row_len, outlier_cap)
        if need <= 0:
            raise ValueError(f"page format {fmt} cannot store pages of {tokens_per_page} x {row_len}")
        super().__init__(n_slots, need, device)
        self.format = fmt
        self.outlier_cap = outlier_cap

    def desc(self) -> "_native.TierStoreDesc":
        return _native.TierStoreDesc(self.data.data_ptr(), self.slot_bytes, self.n_slots, self.format,
                                     self.free_stack.data_ptr(), self.free_top.data_ptr())


class KVLayers:
    """Per-layer K/V token pools ([tokens, heads, head_dim] bf16 each), addressed by pointer tables."""

    def __init__(self, k: Sequence[torch.Tensor], v: Sequence[torch.Tensor]):
        if len(k) != len(v) or not k:
            raise ValueError("need the same number (>0) of K and V layer tensors")
        self.k, self.v = list(k), list(v)
        t0 = self.k[0]
        for t in self.k + self.v:
            if t.dtype != torch.bfloat16 or not t.is_contiguous() or t.shape != t0.shape or not t.is_cuda:
                raise ValueError("K/V layers must be contiguous CUDA bf16 tensors of one shape")
            if t.data_ptr() % 16:
                raise ValueError("K/V layer tensors must be 16-byte aligned")
        self.row_len = int(np.prod(t0.shape[1:]))
        dev = t0.device
        self.k_ptrs = torch.tensor([t.data_ptr() for t in self.k], dtype=torch.int64, device=dev)
        self.v_ptrs = torch.tensor([t.data_ptr() for t in self.v], dtype=torch.int64, device=dev)

    @property
    def n_layers(self) -> int:
        return len(self.k)


@dataclass
class StepLists:
    demote: torch.Tensor   # int32 page rows, first counts[0] valid
    promote: torch.Tensor  # int32 page rows, first counts[1] valid
    counts: torch.Tensor   # int32 [2] on the device
    target: torch.Tensor   # int8 desired tier per page
    R: Optional[torch.Tensor]


class BatchMigrator:
    """Policy plan + mixed-tier migration over a DevicePageTable (see the module docstring).

    ``stores`` maps each compressed tier (``Tier.FP8``, ``Tier.INT4``,
    ``Tier.ARCHIVE``) to its :class:`TierStore`; a tier without a store has no
    codec and pages never move there.  ``status[i]`` / ``released[i]`` report
    entry i of the last :meth:`migrate` call (``_native.MIGRATE_*``).
    """

    def __init__(self, table: DevicePageTable, kv: KVLayers, stores: Mapping[int, TierStore],
                 config: ASHKVConfig, codec_keys: Sequence[tuple[int, int]], *, tokens_per_page: int = 16,
                 seed: int = 42, sigma: float = 3.0, keep_scores: bool = False):
        self.table, self.kv, self.cfg = table, kv, config
        self.tokens_per_page, self.seed, self.sigma = tokens_per_page, int(seed), float(sigma)
        self.stores = {int(t): s for t, s in stores.items()}
        self.next_colder, self.next_hotter = controller_tables(codec_keys)
        caps = {s.outlier_cap for s in self.stores.values() if s.format in (_native.PAGE_NBIT4, _native.PAGE_NBIT2)}
        if len(caps) > 1:
            raise ValueError("dithered stores must share one outlier capacity")
        self.outlier_cap = caps.pop() if caps else 0
        descs = (_native.TierStoreDesc * NUM_TIERS)()
        descs[0] = _native.TierStoreDesc(None, 0, 0, _native.PAGE_BF16, None, None)
        for t in range(1, NUM_TIERS):
            s = self.stores.get(t)
            descs[t] = s.desc() if s is not None else _native.TierStoreDesc(None, 0, 0, _native.PAGE_NONE, None, None)
        self._descs = descs
        n, dev = table.n, table.T.device
        self.lists = StepLists(torch.empty(n, dtype=torch.int32, device=dev), torch.empty(n, dtype=torch.int32, device=dev),
                               torch.zeros(2, dtype=torch.int32, device=dev), torch.empty(n, dtype=torch.int8, device=dev),
                               torch.empty(n, dtype=torch.float32, device=dev) if keep_scores else None)
        self._scratch = torch.empty(_native.policy_scratch_ints(n), dtype=torch.int32, device=dev)
        self.status = torch.zeros(n, dtype=torch.int32, device=dev)
        self.released = torch.full((n,), -1, dtype=torch.int32, device=dev)
        self.demote_status = torch.zeros(n, dtype=torch.int32, device=dev)
        self.demote_released = torch.full((n,), -1, dtype=torch.int32, device=dev)
        self.device_status = torch.zeros(1, dtype=torch.int32, device=dev)
        self._side: Optional[torch.cuda.Stream] = None

    def plan(self, pressure) -> StepLists:
        """Score every page, pick desired tiers and build the transition lists (device-resident).
        ``pressure`` is a float, or a one-element float32 CUDA tensor read on the device (e.g.
        the MAX all-reduce of the ranks' pressures), which keeps the step free of host syncs."""
        t, c, L = self.table, self.cfg, self.lists
        if not isinstance(pressure, torch.Tensor):
            pressure = float(pressure)
        _native.policy_step(t.T, t.S, t.N, t.P, t.tier, (c.w_T, c.w_S, c.w_N, c.w_P), pressure, c.theta_high,
                            c.theta_low, c.delta, c.p_emergency, self.next_colder, self.next_hotter, L.R, L.target,
                            L.demote, L.promote, L.counts, self._scratch)
        return L

    def _move(self, lst, count, target, status, released) -> None:
        t, kv = self.table, self.kv
        tgt = self.lists.target if target is None else target
        _native.migrate_pages(t.tier, t.pin, t.layer, t.token_start, t.slot, tgt, lst, count, kv.k_ptrs, kv.v_ptrs,
                              kv.n_layers, self.tokens_per_page, kv.row_len, kv.row_len, self._descs, self.sigma,
                              self.seed, self.outlier_cap, status, released)

    def migrate(self, lst: torch.Tensor, count: torch.Tensor, target: Optional[torch.Tensor] = None) -> None:
        """Move the first ``*count`` pages of ``lst`` to ``target[page]`` (default: the last plan's
        targets), then release the slots they gave up.  ``status`` / ``released`` report the entries."""
        self._move(lst, count, target, self.status, self.released)
        _native.release_slots(self.released, count, lst.numel(), self._descs, self.device_status)

    def demote(self) -> None:
        self.migrate(self.lists.demote, self.lists.counts[0:1])

    def promote(self) -> None:
        self.migrate(self.lists.promote, self.lists.counts[1:2])

    def demote_and_promote(self) -> None:
        """Both lists of the last plan.  With one compressed tier every edge has a BF16 end:
        demotions only take that tier's slots and promotions only give slots back, which are
        released after both lists either way, so the two lists are moved concurrently on two
        streams.  With more tiers they run in order (a promotion may take a slot a demotion
        released).  ``demote_status`` / ``demote_released`` report the demotion list,
        ``status`` / ``released`` the promotion list."""
        L = self.lists
        if len(self.stores) != 1:
            self._move(L.demote, L.counts[0:1], None, self.demote_status, self.demote_released)
            _native.release_slots(self.demote_released, L.counts[0:1], L.demote.numel(), self._descs,
                                  self.device_status)
            self.promote()
            return
        dev = self.table.T.device
        cur = torch.cuda.current_stream(dev)
        if self._side is None:
            self._side = torch.cuda.Stream(dev)
        self._side.wait_stream(cur)
        with torch.cuda.stream(self._side):
            self._move(L.promote, L.counts[1:2], None, self.status, self.released)
        self._move(L.demote, L.counts[0:1], None, self.demote_status, self.demote_released)
        cur.wait_stream(self._side)
        _native.release_slots(self.demote_released, L.counts[0:1], L.demote.numel(), self._descs, self.device_status)
        _native.release_slots(self.released, L.counts[1:2], L.promote.numel(), self._descs, self.device_status)

    def step(self, pressure) -> StepLists:
        """plan -> demote -> promote, all on the device."""
        L = self.plan(pressure)
        self.demote_and_promote()
        return L

    def pressure(self) -> torch.Tensor:
        """Occupied fraction of the most occupied store, as a one-element device tensor."""
        ps = [s.pressure_tensor() for s in self.stores.values()]
        return torch.stack(ps).max().reshape(1) if ps else torch.zeros(1, device=self.table.T.device)

    def live_slots(self, tier: int) -> int:
        return int(((self.table.tier == tier) & (self.table.slot >= 0)).sum())

    def sync_tiers_to_host(self, page_table: PageTable) -> None:
        """Copy the device tiers back into the host PageTable (row order of ``from_host``)."""
        tiers = self.table.tier.cpu().numpy()
        page_table.columns()["tier"][:] = tiers


class StepGraph:
    """A migration step captured once in a CUDA graph and replayed.

    ``body`` issues the step's device work on the current stream (for a
    tensor-parallel step: the pressure exchange, then ``plan`` with the
    exchanged device pressure, ``demote``, ``promote``).  Replaying the graph
    launches every kernel of the step at once, so the small policy kernels do
    not wait on the host between launches.  Every tensor the body reads must
    keep its address between replays (update pressure inputs in place).
    Construction runs ``body`` once on a side stream first (any one-time
    set-up), which performs a real step: bring the page table back to the
    wanted state before the first replay.
    """

    def __init__(self, body, device: torch.device):
        self.body, self.device = body, device
        side = torch.cuda.Stream(device)
        side.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(side):
            body()
        torch.cuda.current_stream(device).wait_stream(side)
        torch.cuda.synchronize(device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            body()

    def replay(self) -> None:
        self.graph.replay()

    def release(self) -> None:
        """Drop the graph (before the process group that its collectives use is destroyed)."""
        self.graph = None


class Int8PageCodec:
    """Raw BF16 <-> INT8 page kernels over one SlotArena (``ashkv_int8_encode_pages`` /
    ``ashkv_int8_decode_pages``).

    The caller owns the tiers: listed pages must be BF16 pages of valid layers
    without a slot (encode) or pages holding a slot (decode).  ``status_encode[i]``
    / ``status_decode[i]`` report list entry i: 0 ok, 1 no free slot, 2 bad page
    or slot (an encode entry with status 2 leaves its stack slot popped; the
    mixed-tier :class:`BatchMigrator` takes slots only for pages that move).
    """

    def __init__(self, table: DevicePageTable, kv: KVLayers, arena: SlotArena, *, tokens_per_page: int = 16):
        self.table, self.kv, self.arena = table, kv, arena
        self.tokens_per_page = tokens_per_page
        need = int(_native.lib().ashkv_int8_page_slot_bytes(tokens_per_page, kv.row_len))
        if arena.slot_bytes < need:
            raise ValueError(f"arena slots of {arena.slot_bytes} bytes cannot hold a page ({need} bytes)")
        n, dev = table.n, table.T.device
        self.status_encode = torch.zeros(n, dtype=torch.int32, device=dev)
        self.status_decode = torch.zeros(n, dtype=torch.int32, device=dev)

    def _pages_args(self, lst: torch.Tensor, count: torch.Tensor):
        t, kv, a = self.table, self.kv, self.arena
        return (kv.k_ptrs.data_ptr(), kv.v_ptrs.data_ptr(), kv.n_layers, t.layer.data_ptr(), t.token_start.data_ptr(),
                lst.data_ptr(), count.data_ptr(), lst.numel(), self.tokens_per_page, kv.row_len,
                kv.row_len, a.data.data_ptr(), a.slot_bytes, a.n_slots)

    def encode(self, lst: torch.Tensor, count: torch.Tensor) -> None:
        """INT8-encode the first *count pages of ``lst`` into fresh arena slots."""
        a = self.arena
        st = _native.stream_handle(lst.device)
        _native.check(_native.lib().ashkv_int8_encode_pages(
            *self._pages_args(lst, count), a.free_stack.data_ptr(), a.free_top.data_ptr(),
            self.table.slot.data_ptr(), self.status_encode.data_ptr(), st), "int8_encode_pages")
        _native.check(_native.lib().ashkv_slots_commit(count.data_ptr(), lst.numel(), a.free_top.data_ptr(), st),
                      "slots_commit")

    def decode(self, lst: torch.Tensor, count: torch.Tensor, free_slots: bool = True) -> None:
        """Decode the slots of the first *count pages of ``lst`` back into the KV pool."""
        a = self.arena
        _native.check(_native.lib().ashkv_int8_decode_pages(
            *self._pages_args(lst, count), self.table.slot.data_ptr(), int(free_slots), a.free_stack.data_ptr(),
            a.free_top.data_ptr(), self.status_decode.data_ptr(), _native.stream_handle(lst.device)),
            "int8_decode_pages")


def int8_page_slot_bytes(tokens_per_page: int, row_len: int) -> int:
    return int(_native.lib().ashkv_int8_page_slot_bytes(tokens_per_page, row_len))


def stores_for(table: Mapping[tuple[int, int], object], n_slots: Mapping[int, int], device: torch.device,
               tokens_per_page: int, row_len: int, outlier_cap: int = 512) -> dict[int, TierStore]:
    """One TierStore per compressed tier of a resolved codec table (``resolve_codecs``)."""
    from ..compiler.codec_resolver import tier_formats
    out = {}
    for tier, fmt in tier_formats(dict(table)).items():
        if tier == int(Tier.BF16) or fmt < 0 or tier not in n_slots:
            continue
        cap = outlier_cap if fmt in (_native.PAGE_NBIT4, _native.PAGE_NBIT2) else 0
        out[tier] = TierStore(fmt, n_slots[tier], device, tokens_per_page, row_len, cap)
    return out


__all__ = ["DevicePageTable", "SlotArena", "TierStore", "KVLayers", "BatchMigrator", "StepGraph", "Int8PageCodec",
           "StepLists",
           "int8_page_slot_bytes", "stores_for", "Tier"]
