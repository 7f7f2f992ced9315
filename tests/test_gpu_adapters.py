"""GPU tests: SGLang hooks, shadow allocator and batched page migration.

Byte formats are compared with the oracle: the host slot of (token t, layer
l) must hold [fp16 scales of tokens t*H..t*H+H-1 | int8 codes of token t |
zeros], as the reference's hooks write it (with compact host slots, the
zero tail is not transferred and keeps the host pool's previous bytes).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from conftest import assert_int8_codes, assert_int8_roundtrip

from ashkv.adapters.sglang.allocator import SGLangShadowAllocator
from ashkv.adapters.sglang.hooks import SGLangHooks
from ashkv.contracts import ASHKVConfig, Tier
from ashkv import _native
from ashkv.runtime.batch import (BatchMigrator, DevicePageTable, Int8PageCodec, KVLayers, SlotArena, TierStore,
                                int8_page_slot_bytes)

pytestmark = pytest.mark.gpu


def u16(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


class DevicePool:
    def __init__(self, layer_num, capacity, head_num, head_dim, device, seed=0):
        self.layer_num, self.capacity, self.head_num, self.head_dim = layer_num, capacity, head_num, head_dim
        g = torch.Generator(device=device).manual_seed(seed)
        self.k_buffer = [torch.randn(capacity, head_num, head_dim, generator=g, device=device).to(torch.bfloat16)
                         for _ in range(layer_num)]
        self.v_buffer = [torch.randn(capacity, head_num, head_dim, generator=g, device=device).to(torch.bfloat16)
                         for _ in range(layer_num)]


class HostPool:
    def __init__(self, layer_num, capacity, head_num, head_dim, pin=False):
        shape = (capacity, layer_num, head_num, head_dim)
        self.k_buffer = torch.full(shape, 7.0, dtype=torch.bfloat16).pin_memory() if pin else \
            torch.full(shape, 7.0, dtype=torch.bfloat16)
        self.v_buffer = torch.full(shape, 7.0, dtype=torch.bfloat16).pin_memory() if pin else \
            torch.full(shape, 7.0, dtype=torch.bfloat16)
        self.layer_num, self.head_num, self.head_dim = layer_num, head_num, head_dim


def expected_slots(k_layer: torch.Tensor, didx: torch.Tensor, H: int, D: int):
    """Oracle bytes of the host slots [n, 2*H*D] for one layer of K (or V), and a
    mask of the code bytes at tie-zone elements (see conftest.assert_int8_codes)."""
    n, row = didx.numel(), H * D
    rows = u16(k_layer.view(-1, row)[didx.long()]).reshape(n, row)
    codes, scales, tie = oracle.int8_encode(rows, row, scale_fp16=True, with_ties=True)
    out = np.zeros((n, 2 * row), dtype=np.uint8)
    out[:, 2 * H:2 * H + row] = codes.view(np.uint8)
    flat = np.zeros(n * H, dtype=np.uint16)  # slot t carries scales of tokens t*H .. t*H+H-1
    flat[:n] = scales
    out[:, :2 * H] = flat.view(np.uint8).reshape(n, 2 * H)
    ties = np.zeros((n, 2 * row), dtype=bool)
    ties[:, 2 * H:2 * H + row] = tie
    return out, ties


def assert_slots(got: np.ndarray, want: np.ndarray, ties: np.ndarray, what=None) -> None:
    """Slot bytes equal, except INT8 code bytes one apart at tie-zone elements."""
    diff = got != want
    near = np.abs(got.view(np.int8).astype(np.int16) - want.view(np.int8).astype(np.int16)) == 1
    assert not np.any(diff & ~(ties & near)), what


def decoded_rows(slots: np.ndarray, n: int, H: int, D: int) -> np.ndarray:
    """Oracle decode of the codes and scales actually stored in host slots [n, >= 2H + H*D]."""
    flat = slots[:, :2 * H].copy().view(np.uint16).reshape(-1)[:n]
    return oracle.int8_decode(slots[:, 2 * H:2 * H + H * D].copy().view(np.int8), flat, scale_fp16=True)


@pytest.mark.parametrize("compact", [True, False])
@pytest.mark.parametrize("contiguous,pin", [(True, True), (True, False), (False, False), (False, True)])
def test_demote_writes_reference_slot_bytes(cuda, tmp_path, monkeypatch, contiguous, pin, compact):
    monkeypatch.chdir(tmp_path)
    L, cap, H, D, n = 3, 300, 8, 128, 77
    dev = DevicePool(L, cap, H, D, cuda, seed=1)
    host = HostPool(L, cap, H, D, pin=pin)
    before = host.k_buffer.view(cap, L, -1).view(torch.uint8).clone()
    didx = torch.randperm(cap, generator=torch.Generator().manual_seed(2))[:n].to(cuda)
    hidx = torch.arange(10, 10 + n) if contiguous else torch.randperm(cap, generator=torch.Generator().manual_seed(3))[:n]
    hooks = SGLangHooks()
    hooks.compact_host_slots = compact
    assert hooks.demote_hook(dev, host, hidx, didx, "MHA") is True
    used = 2 * H + H * D
    for name in ("k_buffer", "v_buffer"):
        hb = getattr(host, name).view(cap, L, -1).view(torch.uint8)
        for layer in range(L):
            got = hb[hidx.long(), layer].numpy()
            want, ties = expected_slots(getattr(dev, name)[layer], didx, H, D)
            if compact:
                assert_slots(got[:, :used], want[:, :used], ties[:, :used], (name, layer))
                assert np.array_equal(got[:, used:], before[hidx.long(), layer, used:].numpy())
            else:
                assert_slots(got, want, ties, (name, layer))
    slot_bytes = used if compact else 2 * H * D
    assert hooks.transfer_stats["d2h_bytes"] == 2 * n * L * slot_bytes
    # untouched host rows keep their contents
    others = np.setdiff1d(np.arange(cap), hidx.numpy())
    assert bool((host.k_buffer[torch.from_numpy(others)] == 7.0).all())
    # stats: the reference's byte math
    assert hooks.stats["tokens_compressed"] == n * L
    assert hooks.stats["bytes_saved"] == n * L * H * D * 4 - n * L * (H * D + 2 * H) * 2


def test_demote_promote_roundtrip_matches_oracle(cuda, tmp_path, monkeypatch):
    monkeypatch.chdir(tmp_path)
    L, cap, H, D, n = 2, 1000, 32, 128, 500  # the reference GPU test's shapes
    dev = DevicePool(L, cap, H, D, cuda, seed=4)
    host = HostPool(L, cap, H, D)
    didx = torch.arange(n, device=cuda)
    hidx = torch.arange(n)
    orig = [t.clone() for t in dev.k_buffer]
    hooks = SGLangHooks()
    hooks.compressible_layers = [0, 1]
    hooks.demote_hook(dev, host, hidx, didx, "MHA")
    dev.k_buffer[0].zero_()
    assert hooks.promote_hook(dev, host, hidx, didx, 0, "MHA") is True
    restored = dev.k_buffer[0][didx]
    cos = torch.nn.functional.cosine_similarity(orig[0][:n].float().view(1, -1), restored.float().view(1, -1)).item()
    assert cos > 0.99
    slots = host.k_buffer.view(cap, L, -1).view(torch.uint8)[hidx, 0].numpy()
    want_slots, ties = expected_slots(orig[0], didx, H, D)
    assert_slots(slots[:, :2 * H + H * D], want_slots[:, :2 * H + H * D], ties[:, :2 * H + H * D])
    assert np.array_equal(u16(restored).reshape(n, H * D), decoded_rows(slots, n, H, D))
    assert hooks.stats["tokens_decompressed"] == n


@pytest.mark.parametrize("pin,heads", [(False, 8), (True, 8), (True, 1)])
def test_promote_subset_in_reference_order(cuda, tmp_path, monkeypatch, pin, heads):
    """Promote into different device rows with a non-contiguous host index list (a pinned
    host pool takes the indexed gather kernel; 1 head leaves 130-byte slots, padded to 16)."""
    monkeypatch.chdir(tmp_path)
    L, cap, H, D, n = 2, 200, heads, 128, 40
    dev = DevicePool(L, cap, H, D, cuda, seed=5)
    host = HostPool(L, cap, H, D, pin=pin)
    didx = torch.arange(n, device=cuda)
    hidx = torch.randperm(cap, generator=torch.Generator().manual_seed(6))[:n]
    hooks = SGLangHooks()
    src = dev.v_buffer[1][:n].clone()
    hooks.demote_hook(dev, host, hidx, didx, "MHA")
    tgt = torch.arange(100, 100 + n, device=cuda)
    hooks.promote_hook(dev, host, hidx, tgt, 1, "MHA")
    slots = host.v_buffer.view(cap, L, -1).view(torch.uint8)[hidx, 1].numpy()
    want_slots, ties = expected_slots(src, torch.arange(n, device=cuda), H, D)
    used = 2 * H + H * D
    assert_slots(slots[:, :used], want_slots[:, :used], ties[:, :used])
    assert np.array_equal(u16(dev.v_buffer[1][100:100 + n]).reshape(n, H * D), decoded_rows(slots, n, H, D))


def test_hooks_decline_and_native_layers(cuda, tmp_path, monkeypatch):
    monkeypatch.chdir(tmp_path)
    L, cap, H, D, n = 2, 64, 4, 128, 16
    dev = DevicePool(L, cap, H, D, cuda, seed=7)
    host = HostPool(L, cap, H, D)
    idx = torch.arange(n)
    hooks = SGLangHooks()
    assert hooks.demote_hook(dev, host, idx, idx.to(cuda), "MLA") is False
    assert hooks.demote_hook(dev, host, idx[:0], idx[:0].to(cuda), "MHA") is False
    assert hooks.promote_hook(dev, host, idx, idx.to(cuda), 0, "MLA") is False
    hooks.compressible_layers = [0]  # layer 1 travels as plain bf16
    hooks.demote_hook(dev, host, idx, idx.to(cuda), "MHA")
    assert torch.equal(host.k_buffer[:n, 1].view(torch.int16), dev.k_buffer[1][:n].cpu().view(torch.int16))
    used = 2 * H + H * D  # layer 0 compact, layer 1 whole bf16 rows
    got0 = host.k_buffer.view(cap, L, -1).view(torch.uint8)[:n, 0, :used].numpy()
    want0, ties0 = expected_slots(dev.k_buffer[0], idx.to(cuda), H, D)
    assert_slots(got0, want0[:, :used], ties0[:, :used])
    assert hooks.transfer_stats["d2h_bytes"] == 2 * n * (used + 2 * H * D)
    # the same mixed layout through a non-contiguous host index list
    perm = n + torch.randperm(cap - n, generator=torch.Generator().manual_seed(9))[:n]  # rows other than 0..n-1
    hooks.demote_hook(dev, host, perm, idx.to(cuda), "MHA")
    assert torch.equal(host.v_buffer[perm, 1].view(torch.int16), dev.v_buffer[1][:n].cpu().view(torch.int16))
    got0 = host.v_buffer.view(cap, L, -1).view(torch.uint8)[perm, 0, :used].numpy()
    want0, ties0 = expected_slots(dev.v_buffer[0], idx.to(cuda), H, D)
    assert_slots(got0, want0[:, :used], ties0[:, :used])
    saved = dev.k_buffer[1][:n].clone()
    dev.k_buffer[1].zero_()
    hooks.promote_hook(dev, host, idx, idx.to(cuda), 1, "MHA")
    assert torch.equal(dev.k_buffer[1][:n].view(torch.int16), saved.view(torch.int16))


def test_shadow_allocator_arena(cuda):
    a = SGLangShadowAllocator(max_bytes=1 << 20, device=cuda)
    h1 = a.alloc(Tier.FP8, 1000)
    h2 = a.alloc(Tier.FP8, 5000)
    assert h1 > 0 and h2 > 0 and a.pressure() == pytest.approx(6000 / (1 << 20))
    a.write(h1, b"hello world")
    assert a.read(h1)[:11] == b"hello world"
    t = a.get_tensor(h2)
    assert t.is_cuda and t.numel() == 5000 and t.dtype == torch.uint8
    t.fill_(3)
    assert a.read(h2) == b"\x03" * 5000
    offs = a.offsets([h1, h2]).cpu().numpy()
    assert offs[0] % 256 == 0 and offs[1] % 256 == 0 and offs[0] != offs[1]
    assert a.alloc(Tier.FP8, 1 << 20) == -1  # past the budget
    a.free(h1)
    h3 = a.alloc(Tier.FP8, 1000)  # exact-size reuse
    assert a.offsets([h3]).item() == offs[0]
    assert a.read(12345) == b"" and a.get_tensor(12345) is None
    a.free(12345)


@pytest.mark.parametrize("heads", [8, 4, 2, 1])
def test_batch_policy_demote_promote_pages(cuda, heads):
    """Config-4 style: score -> tier -> gather+INT8 encode of the demoted pages into the FP8
    tier's store, then decode+scatter back; bytes compared with the oracle per token row."""
    layers, tokens, T = 4, 4096, 16
    pages_per_layer = tokens // T
    g = torch.Generator(device=cuda).manual_seed(11)
    k = [torch.randn(tokens, heads, 128, generator=g, device=cuda).to(torch.bfloat16) for _ in range(layers)]
    v = [torch.randn(tokens, heads, 128, generator=g, device=cuda).to(torch.bfloat16) for _ in range(layers)]
    kv = KVLayers(k, v)
    n = layers * pages_per_layer
    tab = DevicePageTable.empty(n, cuda)
    for name in ("T", "S", "N", "P"):
        getattr(tab, name).copy_(torch.rand(n, generator=g, device=cuda))
    tab.layer.copy_(torch.arange(n, device=cuda) // pages_per_layer)
    tab.token_start.copy_((torch.arange(n, device=cuda) % pages_per_layer) * T)
    store = TierStore(_native.PAGE_INT8, n, cuda, T, kv.row_len)
    keys = [(0, 1), (1, 0), (1, 2), (2, 1)]
    mig = BatchMigrator(tab, kv, {int(Tier.FP8): store}, ASHKVConfig(), keys, keep_scores=True)
    L = mig.plan(0.9)
    nd, npro = L.counts.tolist()
    assert npro == 0 and nd > n // 10
    orig_k = [t.clone() for t in k]
    mig.demote()
    torch.cuda.synchronize()
    assert store.free_count() == n - nd
    assert int(mig.status[:nd].abs().sum()) == 0 and bool((mig.released[:nd] == -1).all())
    rows = L.demote[:nd].long()
    assert bool((tab.slot[rows] >= 0).all()) and bool((tab.tier[rows] == int(Tier.FP8)).all())
    # wipe the pool, then promote the demoted pages back from their slots
    for li in range(layers):
        k[li].zero_(); v[li].zero_()
    back = torch.zeros(n, dtype=torch.int8, device=cuda)
    mig.migrate(L.demote, L.counts[0:1], target=back)
    torch.cuda.synchronize()
    assert store.free_count() == n
    assert int(mig.status[:nd].abs().sum()) == 0 and bool((tab.tier[rows] == 0).all())
    assert int(tab.slot.ne(-1).sum()) == 0
    sample = rows[:: max(1, nd // 50)].cpu().numpy()
    for p in sample:
        li, ts = int(p) // pages_per_layer, (int(p) % pages_per_layer) * T
        src = u16(orig_k[li][ts:ts + T]).reshape(T, -1)
        assert_int8_roundtrip(u16(k[li][ts:ts + T]), src, kv.row_len)
    # pages that were not demoted stay wiped (the promotion touched only listed pages)
    keep = np.setdiff1d(np.arange(n), rows.cpu().numpy())[:5]
    for p in keep:
        li, ts = int(p) // pages_per_layer, (int(p) % pages_per_layer) * T
        assert bool((k[li][ts:ts + T] == 0).all())


@pytest.mark.parametrize("heads,T", [(1, 16), (2, 12), (8, 16)])
def test_batch_pages_many_entries_per_cta(cuda, heads, T):
    """More list entries than 32 x the grid, so every CTA resolves several batches of
    entries (the last one partial); T=12 leaves row passes partly empty; one entry names
    a layer out of range.  Slot bytes (scales, then K and V codes) and the decoded K/V
    rows are compared with the oracle."""
    layers, ppl = 4, 10240
    tokens, n = ppl * T, layers * ppl
    g = torch.Generator(device=cuda).manual_seed(23 + heads)
    k = [torch.randn(tokens, heads, 128, generator=g, device=cuda).to(torch.bfloat16) for _ in range(layers)]
    v = [torch.randn(tokens, heads, 128, generator=g, device=cuda).to(torch.bfloat16) for _ in range(layers)]
    kv = KVLayers(k, v)
    L = kv.row_len
    tab = DevicePageTable.empty(n, cuda)
    idx = torch.arange(n, device=cuda)
    tab.layer.copy_(idx // ppl)
    tab.token_start.copy_((idx % ppl) * T)
    bad = n // 3
    tab.layer[bad] = layers
    sb = int8_page_slot_bytes(T, L)
    arena = SlotArena(n, sb, cuda)
    mig = Int8PageCodec(tab, kv, arena, tokens_per_page=T)
    lst = torch.randperm(n, generator=g, device=cuda).to(torch.int32)
    cnt = torch.tensor([n], dtype=torch.int32, device=cuda)
    orig = [[t.clone() for t in k], [t.clone() for t in v]]
    mig.encode(lst, cnt)
    torch.cuda.synchronize()
    pos_bad = int((lst == bad).nonzero()[0, 0])
    st = mig.status_encode[:n].cpu().numpy()
    assert st[pos_bad] == 2 and int(np.count_nonzero(st)) == 1
    assert arena.free_count() == 0
    slot = tab.slot.cpu().numpy()
    assert slot[bad] == -1 and len(np.unique(np.delete(slot, bad))) == n - 1
    c0 = (4 * T + 15) // 16 * 16
    sample = np.unique(np.r_[np.arange(0, n, n // 97), n - 1])
    sample = sample[sample != bad]
    blobs = arena.data.view(n, sb)[torch.from_numpy(slot[sample]).long().to(cuda)].cpu().numpy()
    for p, blob in zip(sample, blobs):
        li, ts = int(p) // ppl, (int(p) % ppl) * T
        sc = blob[:4 * T].view(np.uint16)
        for h in range(2):
            codes, scales, tie = oracle.int8_encode(u16(orig[h][li][ts:ts + T]).reshape(T, L), L, scale_fp16=True,
                                                    with_ties=True)
            assert np.array_equal(sc[h * T:(h + 1) * T], scales)
            assert_int8_codes(blob[c0 + h * T * L:c0 + (h + 1) * T * L].view(np.int8).reshape(T, L), codes, tie)
    for t in k + v:
        t.zero_()
    mig.decode(lst, cnt, free_slots=True)
    torch.cuda.synchronize()
    sd = mig.status_decode[:n].cpu().numpy()
    assert sd[pos_bad] == 2 and int(np.count_nonzero(sd)) == 1
    assert arena.free_count() == n - 1
    assert int(tab.slot.ne(-1).sum()) == 0
    rows = tokens if heads <= 2 else 2048  # whole layers through the oracle for narrow rows
    for h, cur in enumerate((k, v)):
        for li in range(layers):
            got = u16(cur[li][:rows]).reshape(rows, L)
            src = u16(orig[h][li][:rows]).reshape(rows, L)
            if li == bad // ppl:
                b0 = (bad % ppl) * T
                assert not got[b0:b0 + T].any()
                got, src = np.delete(got, np.s_[b0:b0 + T], 0), np.delete(src, np.s_[b0:b0 + T], 0)
            assert_int8_roundtrip(got, src, L)


@pytest.mark.parametrize("heads", [1, 8])
def test_batch_pages_nan_inf_rows_match_oracle(cuda, heads):
    """Token rows holding NaN, +-inf, all-NaN and all-zero values: slot bytes equal the oracle's."""
    T, ppl = 16, 8
    tokens = T * ppl
    g = torch.Generator(device=cuda).manual_seed(41)
    k = torch.randn(tokens, heads, 128, generator=g, device=cuda).to(torch.bfloat16)
    v = torch.randn(tokens, heads, 128, generator=g, device=cuda).to(torch.bfloat16)
    kb, vb = k.view(torch.int16).view(tokens, -1), v.view(torch.int16).view(tokens, -1)
    kb[0, 0] = 0x7FC0
    kb[1, 5] = 0xFF80 - 0x10000     # -inf (0xFF80) as int16
    kb[2, :] = 0x7FC0
    kb[3, :] = 0
    vb[4, 7] = 0x7FA0
    vb[5, 1], vb[5, 2] = 0x7F80, 0x7FC0
    kv = KVLayers([k], [v])
    L = kv.row_len
    tab = DevicePageTable.empty(ppl, cuda)
    tab.token_start.copy_(torch.arange(ppl, device=cuda, dtype=torch.int32) * T)
    sb = int8_page_slot_bytes(T, L)
    arena = SlotArena(ppl, sb, cuda)
    mig = Int8PageCodec(tab, kv, arena)
    lst = torch.arange(ppl, dtype=torch.int32, device=cuda)
    mig.encode(lst, torch.tensor([ppl], dtype=torch.int32, device=cuda))
    torch.cuda.synchronize()
    assert int(mig.status_encode[:ppl].abs().sum()) == 0
    slot = tab.slot.cpu().numpy()
    data = arena.data.view(ppl, sb).cpu().numpy()
    c0 = (4 * T + 15) // 16 * 16
    for p in range(ppl):
        blob = data[slot[p]]
        for h, t in enumerate((k, v)):
            codes, scales, tie = oracle.int8_encode(u16(t[p * T:(p + 1) * T]).reshape(T, L), L, scale_fp16=True,
                                                    with_ties=True)
            assert np.array_equal(blob[:4 * T].view(np.uint16)[h * T:(h + 1) * T], scales), (p, h)
            assert_int8_codes(blob[c0 + h * T * L:c0 + (h + 1) * T * L].view(np.int8).reshape(T, L), codes, tie)


def test_batch_encode_runs_out_of_slots(cuda):
    layers, tokens, T = 1, 1024, 16
    kv = KVLayers([torch.randn(tokens, 8, 128, device=cuda).to(torch.bfloat16)],
                  [torch.randn(tokens, 8, 128, device=cuda).to(torch.bfloat16)])
    n = tokens // T
    tab = DevicePageTable.empty(n, cuda)
    tab.token_start.copy_(torch.arange(n, device=cuda, dtype=torch.int32) * T)
    arena = SlotArena(10, int8_page_slot_bytes(T, kv.row_len), cuda)
    mig = Int8PageCodec(tab, kv, arena)
    lst = torch.arange(n, dtype=torch.int32, device=cuda)
    cnt = torch.tensor([n], dtype=torch.int32, device=cuda)
    mig.encode(lst, cnt)
    st = mig.status_encode[:n].cpu().numpy()
    assert (st[:10] == 0).all() and (st[10:] == 1).all()
    assert arena.free_count() == 0
