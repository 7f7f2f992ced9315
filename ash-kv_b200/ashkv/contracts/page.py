"""Page metadata table.

Same public surface and never-raise semantics as ``PageTable`` in
ashkv/contracts/page.py:63-295 of the reference: a numpy structured array
(``PAGE_DTYPE``, identical field names, types and order, because
``snapshot()`` consumers index it by field), an O(1) page_id -> row map,
swap-with-last removal, and ``apply_tier_transition`` as the only hot-path
mutator, which refuses pinned pages.

The GPU policy path reads the same columns through
``ashkv.runtime.device_table.DevicePageTable``.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from .tiers import Tier

PAGE_DTYPE = np.dtype([
    ("page_id", np.int64),
    ("layer_id", np.int32),
    ("token_start", np.int32),
    ("token_end", np.int32),
    ("tier", np.int8),
    ("pin_count", np.int32),
    ("last_access", np.int64),
    ("access_count", np.int64),
    ("creation_time", np.int64),
    ("bf16_checksum", np.uint64),
    ("current_checksum", np.uint64),
    ("T", np.float32),
    ("S", np.float32),
    ("N", np.float32),
    ("P", np.float32),
])


@dataclass(slots=True, frozen=True)
class PageHandle:
    page_id: int


class PageTable:
    """Numpy-backed page metadata; not thread-safe (one caller per decode step)."""

    __slots__ = ("_arr", "_next_id", "_page_to_row", "_capacity", "_size")

    def __init__(self, capacity: int = 1 << 20) -> None:
        self._capacity = int(capacity)
        self._arr = np.zeros(self._capacity, dtype=PAGE_DTYPE)
        self._arr["page_id"] = -1
        self._next_id = 0
        self._size = 0
        self._page_to_row = np.full(max(2 * self._capacity, 1024), -1, dtype=np.int64)

    # -- internal ------------------------------------------------------------
    def _row(self, page_id: int) -> int:
        if 0 <= page_id < self._page_to_row.shape[0]:
            return int(self._page_to_row[page_id])
        return -1

    def _grow_map(self, page_id: int) -> None:
        n = self._page_to_row.shape[0]
        if page_id < n:
            return
        grown = np.full(max(2 * n, page_id + 1024), -1, dtype=np.int64)
        grown[:n] = self._page_to_row
        self._page_to_row = grown

    # -- cold path: lifecycle --------------------------------------------------
    def add(self, layer_id: int, token_start: int, token_end: int, bf16_checksum: int,
            creation_time: int) -> int:
        """Register a page at BF16 with T=1.0; raises RuntimeError when full."""
        if self._size >= self._capacity:
            raise RuntimeError(f"PageTable full (capacity={self._capacity})")
        row, pid = self._size, self._next_id
        self._next_id += 1
        self._size += 1
        r = self._arr[row]
        r["page_id"] = pid
        r["layer_id"] = layer_id
        r["token_start"] = token_start
        r["token_end"] = token_end
        r["tier"] = int(Tier.BF16)
        r["pin_count"] = 0
        r["last_access"] = creation_time
        r["access_count"] = 0
        r["creation_time"] = creation_time
        r["bf16_checksum"] = bf16_checksum
        r["current_checksum"] = bf16_checksum
        r["T"], r["S"], r["N"], r["P"] = 1.0, 0.0, 0.0, 0.0
        self._grow_map(pid)
        self._page_to_row[pid] = row
        return pid

    def add_many(self, layer_id: np.ndarray, token_start: np.ndarray, token_end: np.ndarray,
                 bf16_checksum: np.ndarray, creation_time: int = 0) -> np.ndarray:
        """Vectorised ``add`` for bulk registration; returns the new page ids."""
        n = int(len(layer_id))
        if self._size + n > self._capacity:
            raise RuntimeError(f"PageTable full (capacity={self._capacity})")
        rows = np.arange(self._size, self._size + n)
        pids = np.arange(self._next_id, self._next_id + n, dtype=np.int64)
        a = self._arr
        a["page_id"][rows] = pids
        a["layer_id"][rows] = layer_id
        a["token_start"][rows] = token_start
        a["token_end"][rows] = token_end
        a["tier"][rows] = int(Tier.BF16)
        a["pin_count"][rows] = 0
        a["last_access"][rows] = creation_time
        a["access_count"][rows] = 0
        a["creation_time"][rows] = creation_time
        a["bf16_checksum"][rows] = bf16_checksum
        a["current_checksum"][rows] = bf16_checksum
        a["T"][rows], a["S"][rows], a["N"][rows], a["P"][rows] = 1.0, 0.0, 0.0, 0.0
        self._grow_map(int(pids[-1]) if n else 0)
        self._page_to_row[pids] = rows
        self._next_id += n
        self._size += n
        return pids

    def remove(self, page_id: int) -> None:
        row = self._row(page_id)
        if row < 0:
            return
        self._page_to_row[page_id] = -1
        last = self._size - 1
        if row != last:
            self._arr[row] = self._arr[last]
            self._page_to_row[int(self._arr[row]["page_id"])] = row
        self._size -= 1

    # -- hot path: read ------------------------------------------------------------
    def snapshot(self) -> np.ndarray:
        return self._arr[: self._size].copy()

    def columns(self) -> np.ndarray:
        """Zero-copy view of the active rows (for uploads to the device mirror)."""
        return self._arr[: self._size]

    def find(self, page_id: int) -> int:
        return self._row(page_id)

    def get_tier(self, page_id: int) -> int:
        row = self._row(page_id)
        return -1 if row < 0 else int(self._arr["tier"][row])

    def get_pin_count(self, page_id: int) -> int:
        row = self._row(page_id)
        return -1 if row < 0 else int(self._arr["pin_count"][row])

    def get_bf16_checksum(self, page_id: int) -> int:
        row = self._row(page_id)
        return 0 if row < 0 else int(self._arr["bf16_checksum"][row])

    @property
    def size(self) -> int:
        return self._size

    def __len__(self) -> int:
        return self._size

    # -- hot path: transitions -----------------------------------------------------
    def apply_tier_transition(self, page_id: int, new_tier: Tier, new_checksum: int) -> bool:
        row = self._row(page_id)
        if row < 0 or self._arr["pin_count"][row] > 0:
            return False
        self._arr["tier"][row] = int(new_tier)
        self._arr["current_checksum"][row] = new_checksum
        return True

    def apply_tier_transitions(self, rows: np.ndarray, new_tiers: np.ndarray,
                               new_checksums: np.ndarray) -> np.ndarray:
        """Vectorised commit by row index; returns the mask of rows committed (unpinned)."""
        rows = np.asarray(rows, dtype=np.int64)
        ok = (rows >= 0) & (rows < self._size)
        ok[ok] = self._arr["pin_count"][rows[ok]] <= 0
        sel = rows[ok]
        self._arr["tier"][sel] = np.asarray(new_tiers)[ok]
        self._arr["current_checksum"][sel] = np.asarray(new_checksums)[ok]
        return ok

    # -- cold path: metadata -------------------------------------------------------
    def touch(self, page_id: int, time: int) -> None:
        row = self._row(page_id)
        if row < 0:
            return
        self._arr["last_access"][row] = time
        self._arr["access_count"][row] += 1

    def pin(self, page_id: int) -> None:
        row = self._row(page_id)
        if row >= 0:
            self._arr["pin_count"][row] += 1

    def unpin(self, page_id: int) -> None:
        row = self._row(page_id)
        if row >= 0 and self._arr["pin_count"][row] > 0:
            self._arr["pin_count"][row] -= 1

    def update_score_inputs(self, page_ids: np.ndarray, T: np.ndarray, S: np.ndarray, N: np.ndarray,
                            P: np.ndarray) -> None:
        n = len(page_ids)
        if not (len(T) == len(S) == len(N) == len(P) == n):
            return
        page_ids = np.asarray(page_ids)
        inside = (page_ids >= 0) & (page_ids < self._page_to_row.shape[0])
        rows = np.full(n, -1, dtype=np.int64)
        rows[inside] = self._page_to_row[page_ids[inside]]
        ok = rows >= 0
        if not ok.any():
            return
        r = rows[ok]
        self._arr["T"][r] = np.asarray(T)[ok]
        self._arr["S"][r] = np.asarray(S)[ok]
        self._arr["N"][r] = np.asarray(N)[ok]
        self._arr["P"][r] = np.asarray(P)[ok]
