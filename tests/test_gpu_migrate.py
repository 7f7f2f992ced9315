"""GPU tests: mixed-tier batched migration (ashkv_migrate_pages / ashkv_release_slots).

Every tier edge the controller plans runs the codec of its tier on the
device.  Parity: a page placed in a source tier (slot bytes written from the
oracle) and migrated must land in the target tier as the oracle's encode of
the oracle's decode of those bytes: bit-exact for every format, INT8 codes
one apart only at tie-zone elements (see ``conftest.assert_int8_codes``).
The per-entry ladder follows migrate() (ashkv/runtime/migrate.py:93-145):
pinned, already at target, no codec, bad page, no slot; a dithered page with
more outliers than its slot holds stays where it is.  Slots are accounted
exactly over repeated policy steps with pinned pages.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle

from ashkv import _native
from ashkv.contracts import ASHKVConfig, Tier
from ashkv.runtime.batch import BatchMigrator, DevicePageTable, KVLayers, TierStore

pytestmark = pytest.mark.gpu

BF16, INT8, FP8, INT4, NBIT4, NBIT2 = (_native.PAGE_BF16, _native.PAGE_INT8, _native.PAGE_FP8, _native.PAGE_INT4,
                                       _native.PAGE_NBIT4, _native.PAGE_NBIT2)
NBIT = (NBIT4, NBIT2)
KEYS_ALL = [(0, 1), (1, 0), (1, 2), (2, 1), (2, 3), (3, 2)]
SEED, CAP = 1234, 512


def u16(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


class Env:
    """A KV pool of n pages (2 layers, T tokens of `heads` x 128) with its page table."""

    def __init__(self, cuda, n: int, T: int, heads: int, seed: int = 0, outlier_frac: float = 0.001):
        self.n, self.T, self.dev = n, T, cuda
        self.layers = 2
        self.ppl = n // self.layers
        g = torch.Generator(device=cuda).manual_seed(seed)
        shape = (self.ppl * T, heads, 128)

        def pool():
            x = torch.randn(shape, generator=g, device=cuda)
            x = torch.where(torch.rand(shape, generator=g, device=cuda) < outlier_frac, x * 50.0, x)
            return x.to(torch.bfloat16)
        self.k = [pool() for _ in range(self.layers)]
        self.v = [pool() for _ in range(self.layers)]
        self.kv = KVLayers(self.k, self.v)
        self.row = self.kv.row_len
        self.E = 2 * T * self.row
        self.tab = DevicePageTable.empty(n, cuda)
        idx = torch.arange(n, device=cuda)
        self.tab.layer.copy_(idx // self.ppl)
        self.tab.token_start.copy_((idx % self.ppl) * T)

    def page_bits(self, p: int) -> np.ndarray:
        li, ts = p // self.ppl, (p % self.ppl) * self.T
        return np.concatenate([u16(self.k[li][ts:ts + self.T]).reshape(-1), u16(self.v[li][ts:ts + self.T]).reshape(-1)])

    def set_page_bits(self, p: int, bits: np.ndarray) -> None:
        li, ts = p // self.ppl, (p % self.ppl) * self.T
        half = bits.size // 2
        for pool, part in ((self.k[li], bits[:half]), (self.v[li], bits[half:])):
            pool[ts:ts + self.T].view(torch.int16).copy_(
                torch.from_numpy(part.astype(np.uint16).view(np.int16).copy()).view(pool[ts:ts + self.T].shape))


def place(env: Env, store: TierStore, tier: int, pages, slots_bytes) -> None:
    """Write oracle slot bytes for `pages` into slots 0.. of `store` and mark the pages as held there."""
    sv = store.slot_view()
    for j, (p, b) in enumerate(zip(pages, slots_bytes)):
        row = torch.zeros(store.slot_bytes, dtype=torch.uint8)
        row[: b.size] = torch.from_numpy(b)
        sv[j].copy_(row.to(env.dev))
        env.tab.tier[p] = tier
        env.tab.slot[p] = j
    k = len(pages)
    store.free_stack[: store.n_slots - k].copy_(torch.arange(store.n_slots - 1, k - 1, -1, dtype=torch.int32))
    store.free_top.fill_(store.n_slots - k)


def current_bytes(env: Env, mig: BatchMigrator, p: int) -> tuple[int, np.ndarray]:
    """(format, bytes) of page p where it lives now: pool rows, or its slot."""
    t = int(env.tab.tier[p])
    if t == 0:
        return BF16, env.page_bits(p)
    st = mig.stores[t]
    return st.format, st.slot_view()[int(env.tab.slot[p])].cpu().numpy()


def expect_transcode(env: Env, src_fmt: int, src: np.ndarray, dst_fmt: int, p: int):
    """Oracle: bytes of page p in dst_fmt from its bytes in src_fmt (+ tie mask, outlier count)."""
    page = src if src_fmt == BF16 else oracle.page_decode(src_fmt, src, env.T, env.row, outlier_cap=CAP)
    if dst_fmt == BF16:
        return page, np.zeros(page.size, bool), 0
    return oracle.page_encode(dst_fmt, page, env.T, env.row, page_id=p, seed=SEED, outlier_cap=CAP)


def assert_bytes(got: np.ndarray, want: np.ndarray, ties: np.ndarray, what) -> None:
    if want.dtype != np.uint8:  # bf16 pool rows: exact
        assert np.array_equal(got, want), (what, int((got != want).sum()))
        return
    got = got[: want.size]
    diff = got != want
    near = np.abs(got.view(np.int8).astype(np.int16) - want.view(np.int8).astype(np.int16)) == 1
    assert not np.any(diff & ~(ties & near)), (what, int(diff.sum()))


EDGES = [(BF16, INT8), (BF16, FP8), (BF16, INT4), (BF16, NBIT4), (INT8, BF16), (FP8, BF16), (INT8, INT4),
         (INT8, NBIT4), (FP8, INT4), (INT4, INT8), (NBIT4, INT8), (INT4, NBIT2), (NBIT2, INT4), (NBIT2, NBIT4),
         (NBIT4, NBIT2), (NBIT2, BF16), (INT4, FP8), (NBIT4, FP8), (FP8, INT8), (NBIT2, INT8), (INT8, FP8),
         (NBIT4, INT4)]
FMT_NAME = {BF16: "bf16", INT8: "int8", FP8: "fp8", INT4: "int4", NBIT4: "nbit4", NBIT2: "nbit2"}


@pytest.mark.parametrize("heads", [8, 4, 1])
@pytest.mark.parametrize("edge", EDGES, ids=[f"{FMT_NAME[a]}-{FMT_NAME[b]}" for a, b in EDGES])
def test_edge_matches_oracle(cuda, edge, heads):
    src_fmt, dst_fmt = edge
    n = {8: 96, 4: 128, 1: 256}[heads]
    env = Env(cuda, n, 16, heads, seed=7 + src_fmt * 7 + dst_fmt)
    src_tier = 0 if src_fmt == BF16 else 1
    dst_tier = 0 if dst_fmt == BF16 else (2 if src_fmt != BF16 else 1)
    stores = {}
    if src_fmt != BF16:
        stores[src_tier] = TierStore(src_fmt, n, cuda, env.T, env.row, CAP if src_fmt in NBIT else 0)
    if dst_fmt != BF16:
        stores[dst_tier] = TierStore(dst_fmt, n, cuda, env.T, env.row, CAP if dst_fmt in NBIT else 0)
    mig = BatchMigrator(env.tab, env.kv, stores, ASHKVConfig(), KEYS_ALL, seed=SEED)
    pages = list(range(0, n, 1))
    src_bytes = {}
    if src_fmt != BF16:
        made = [oracle.page_encode(src_fmt, env.page_bits(p), env.T, env.row, page_id=p + 77, seed=99,
                                   outlier_cap=CAP)[0] for p in pages]
        place(env, stores[src_tier], src_tier, pages, made)
        src_bytes = dict(zip(pages, made))
    else:
        src_bytes = {p: env.page_bits(p) for p in pages}
    if dst_fmt == BF16:  # the pool rows are overwritten: wipe them so stale values cannot pass
        for t in env.k + env.v:
            t.zero_()
    target = torch.full((n,), dst_tier, dtype=torch.int8, device=cuda)
    lst = torch.tensor(pages, dtype=torch.int32, device=cuda)
    cnt = torch.tensor([len(pages)], dtype=torch.int32, device=cuda)
    mig.migrate(lst, cnt, target=target)
    torch.cuda.synchronize()
    st = mig.status[: len(pages)].cpu().numpy()
    n_out_total = 0
    for j, p in enumerate(pages):
        want, ties, n_out = expect_transcode(env, src_fmt, src_bytes[p], dst_fmt, p)
        n_out_total += n_out
        assert st[j] == _native.MIGRATE_OK, (p, st[j])
        fmt, got = current_bytes(env, mig, p)
        assert fmt == dst_fmt
        assert_bytes(got, want, ties, (edge, p))
    assert int((env.tab.tier == dst_tier).sum()) == n
    if dst_fmt in NBIT:
        assert n_out_total > 0  # the data carries outliers, so the outlier lists are exercised
    # every source slot went back; every destination slot is live exactly once
    if src_fmt != BF16:
        assert stores[src_tier].free_count() == n
    if dst_fmt != BF16:
        assert stores[dst_tier].free_count() == 0
        assert len(np.unique(env.tab.slot.cpu().numpy())) == n


def test_entry_ladder_statuses(cuda):
    """Pinned, already at target, tier without a codec, bad layer, no free slot and
    outlier overflow: each leaves the page where it was and takes no slot."""
    n = 64
    env = Env(cuda, n, 16, 1, seed=3)
    fp8 = TierStore(INT8, 6, cuda, env.T, env.row)
    arch = TierStore(NBIT2, 4, cuda, env.T, env.row, outlier_cap=8)
    mig = BatchMigrator(env.tab, env.kv, {int(Tier.FP8): fp8, int(Tier.ARCHIVE): arch}, ASHKVConfig(), KEYS_ALL,
                        seed=SEED)
    # page 10 gets many outliers: more than 8 beyond 3 sigma
    b = env.page_bits(10).copy()
    vals = (b.astype(np.uint32) << 16).view(np.float32)
    vals[::31] *= 60.0
    env.set_page_bits(10, torch.from_numpy(vals).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16))
    target = torch.full((n,), 1, dtype=torch.int8, device=cuda)
    env.tab.pin[0] = 1                    # pinned
    target[1] = 0                         # already at target (BF16)
    target[2] = 2                         # INT4 tier has no store: no codec
    env.tab.layer[3] = 5                  # bad layer
    target[10] = 3                        # archive: overflow
    lst = torch.tensor([0, 1, 2, 3, 10] + list(range(20, 28)), dtype=torch.int32, device=cuda)
    cnt = torch.tensor([lst.numel()], dtype=torch.int32, device=cuda)
    tiers_before = env.tab.tier.clone()
    mig.migrate(lst, cnt, target=target)
    torch.cuda.synchronize()
    st = mig.status[: lst.numel()].cpu().numpy()
    assert list(st[:5]) == [_native.MIGRATE_PINNED, _native.MIGRATE_SAME_TIER, _native.MIGRATE_NO_CODEC,
                            _native.MIGRATE_BAD_PAGE, _native.MIGRATE_OVERFLOW]
    ok = st[5:] == _native.MIGRATE_OK
    assert ok.sum() == 6 and (st[5:][~ok] == _native.MIGRATE_NO_SLOT).all()
    moved = lst[5:].cpu().numpy()[ok]
    assert bool((env.tab.tier[torch.from_numpy(moved).to(cuda)] == 1).all())
    for p in (0, 1, 2, 3, 10):
        assert int(env.tab.tier[p]) == int(tiers_before[p]) and int(env.tab.slot[p]) == -1
    assert fp8.free_count() == 0 and arch.free_count() == 4  # the overflowed slot came back
    assert int(mig.device_status.item()) == 0


def _place_mixed(env: Env, mig: BatchMigrator, tiers0: np.ndarray) -> None:
    """Bring every page to tiers0[p] by migrations from BF16 (and onward), as in a running engine."""
    n = env.n
    for hop in (1, 2, 3):
        want = np.minimum(tiers0, hop)
        cur = env.tab.tier.cpu().numpy()
        pages = np.nonzero(want > cur)[0].astype(np.int32)
        if pages.size == 0:
            continue
        target = torch.from_numpy(want.astype(np.int8)).to(env.dev)
        lst = torch.from_numpy(pages).to(env.dev)
        mig.migrate(lst, torch.tensor([pages.size], dtype=torch.int32, device=env.dev), target=target)
        torch.cuda.synchronize()
        assert (mig.status[: pages.size].cpu().numpy() == _native.MIGRATE_OK).all()
    assert np.array_equal(env.tab.tier.cpu().numpy(), tiers0.astype(np.int8))


def _check_accounting(env: Env, mig: BatchMigrator) -> None:
    tier = env.tab.tier.cpu().numpy()
    slot = env.tab.slot.cpu().numpy()
    assert (slot[tier == 0] == -1).all()
    for t, s in mig.stores.items():
        live = slot[tier == t]
        assert (live >= 0).all() and len(np.unique(live)) == live.size
        assert s.free_count() + live.size == s.n_slots, (t, s.free_count(), live.size)
        free = s.free_stack[: s.free_count()].cpu().numpy()
        assert len(np.intersect1d(free, live)) == 0 and len(np.unique(free)) == free.size


@pytest.mark.parametrize("tiers", [3, 1])
def test_repeated_steps_account_every_slot(cuda, tiers):
    """Plan -> demote -> promote repeated with changing features, changing pressure and
    pinned pages: no slot is lost or shared, pinned pages never move, and every page that
    moved holds the oracle's transcode of what it held before the step.  With one
    compressed tier the step moves its two lists concurrently."""
    n = 2048
    env = Env(cuda, n, 16, 1, seed=5)
    stores = {1: TierStore(INT8, n, cuda, env.T, env.row)}
    if tiers == 3:
        stores.update({2: TierStore(INT4, n, cuda, env.T, env.row),
                       3: TierStore(NBIT2, n, cuda, env.T, env.row, outlier_cap=CAP)})
    keys = KEYS_ALL if tiers == 3 else [(0, 1), (1, 0)]
    mig = BatchMigrator(env.tab, env.kv, stores, ASHKVConfig(), keys, seed=SEED)
    rng = np.random.default_rng(0)
    _place_mixed(env, mig, rng.integers(0, tiers + 1, n))
    pinned = rng.choice(n, 100, replace=False)
    env.tab.pin[torch.from_numpy(pinned).to(cuda)] = 1
    sample = rng.choice(n, 48, replace=False)
    for step, p in enumerate((0.5, 0.9, 0.97, 0.7, 0.96, 0.95)):
        for name in ("T", "S", "N", "P"):
            getattr(env.tab, name).copy_(torch.from_numpy(rng.random(n, dtype=np.float32)).to(cuda))
        before = {q: current_bytes(env, mig, int(q)) for q in sample}
        tiers_before = env.tab.tier.cpu().numpy()
        L = mig.step(p)
        torch.cuda.synchronize()
        _check_accounting(env, mig)
        tiers = env.tab.tier.cpu().numpy()
        assert np.array_equal(tiers[pinned], tiers_before[pinned])
        assert (np.abs(tiers.astype(int) - tiers_before.astype(int)) <= 1).all()
        nd, npro = L.counts.tolist()
        assert nd + npro > 0
        for q in sample:
            if tiers[q] == tiers_before[q]:
                continue
            src_fmt, src = before[q]
            dst_fmt, got = current_bytes(env, mig, int(q))
            want, ties, _ = expect_transcode(env, src_fmt, src, dst_fmt, int(q))
            assert_bytes(got, want, ties, (step, int(q)))


@pytest.mark.parametrize("pressure", [0.5, 0.7, 0.9, 0.95, 0.96, 0.97])
def test_config5_mixed_tiers_pressure_sweep(cuda, pressure):
    """Config 5 at reduced size: uniform features and tiers {BF16, INT8, INT4, INT2}; the
    plan's lists equal the oracle's desired tiers, and the step commits exactly them."""
    n = 8192
    env = Env(cuda, n, 16, 1, seed=11)
    stores = {1: TierStore(INT8, n, cuda, env.T, env.row), 2: TierStore(INT4, n, cuda, env.T, env.row),
              3: TierStore(NBIT2, n, cuda, env.T, env.row, outlier_cap=CAP)}
    mig = BatchMigrator(env.tab, env.kv, stores, ASHKVConfig(), KEYS_ALL, seed=SEED)
    rng = np.random.default_rng(int(pressure * 100))
    tiers0 = rng.integers(0, 4, n)
    _place_mixed(env, mig, tiers0)
    feats = [rng.random(n, dtype=np.float32) for _ in range(4)]
    for name, f in zip(("T", "S", "N", "P"), feats):
        getattr(env.tab, name).copy_(torch.from_numpy(f).to(cuda))
    c = ASHKVConfig()
    R = oracle.score(*feats, c.w_T, c.w_S, c.w_N, c.w_P)
    nc, nh = oracle.controller_tables(KEYS_ALL)
    want = oracle.desired_tiers(R, tiers0.astype(np.int8), pressure, c.theta_high, c.theta_low, c.delta,
                                c.p_emergency, nc, nh)
    mig.step(pressure)
    torch.cuda.synchronize()
    assert np.array_equal(env.tab.tier.cpu().numpy(), want)
    _check_accounting(env, mig)
