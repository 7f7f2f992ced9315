"""Host-side logic on CPU: contracts, the migrate() ladder under injected
faults, the registry, circuit breakers, hook bookkeeping, the patcher and the
arena allocator's bookkeeping.  No GPU: faults come from mock codecs and
allocators defined here."""
from __future__ import annotations

import json
import os
import sys
import time
import types
from unittest.mock import MagicMock, patch

import numpy as np
import pytest

from ashkv.adapters.sglang import patcher as patcher_mod
from ashkv.adapters.sglang.allocator import SGLangShadowAllocator
from ashkv.adapters.sglang.hooks import SGLangHooks
from ashkv.compiler import CodecRegistry, controller_tables
from ashkv.contracts import (PAGE_DTYPE, ASHKVConfig, Allocator, Codec, MigrationResult, MigrationStatus,
                             PageTable, Tier, next_colder, next_hotter, tier_distance)
from ashkv.runtime import MockAllocator, migrate
from ashkv.safety import CircuitBreaker, CircuitBreakerRegistry

import oracle


# ------------------------------------------------------------------ mocks
class XorCodec:
    """Lossless mock: encode = xor 0x5A, decode = xor back."""

    def __init__(self, fail=None, corrupt=False):
        self.fail, self.corrupt = fail, corrupt

    def encode(self, b):
        if self.fail == "encode":
            raise RuntimeError("injected encode failure")
        return bytes(x ^ 0x5A for x in b)

    def decode(self, b):
        if self.fail == "decode":
            raise RuntimeError("injected decode failure")
        out = bytes(x ^ 0x5A for x in b)
        return out[:-1] + bytes([out[-1] ^ 1]) if self.corrupt and out else out

    def checksum(self, b):
        if self.fail == "checksum":
            raise RuntimeError("injected checksum failure")
        return oracle.xxh64(b)


class FaultyAllocator(MockAllocator):
    """Raises from one method once armed (after the test page is set up)."""

    def __init__(self, fail=None):
        super().__init__()
        self.fail, self.armed = fail, False

    def read(self, h):
        if self.armed and self.fail == "read":
            raise RuntimeError("read")
        return super().read(h)

    def write(self, h, d):
        if self.armed and self.fail == "write":
            raise RuntimeError("write")
        super().write(h, d)

    def alloc(self, t, n):
        if self.armed and self.fail == "alloc":
            raise RuntimeError("alloc")
        return super().alloc(t, n)


def setup_page(alloc, data=b"\x01\x02\x03\x04" * 64):
    pt = PageTable(capacity=16)
    pid = pt.add(layer_id=0, token_start=0, token_end=16, bf16_checksum=oracle.xxh64(data), creation_time=0)
    h = alloc.alloc(Tier.BF16, len(data))
    alloc.write(h, data)
    handles = {pid: h}
    return pt, pid, handles


# ------------------------------------------------------------------ contracts
def test_tiers_and_config():
    assert [int(t) for t in Tier] == [0, 1, 2, 3, 4, 5]
    assert next_hotter(Tier.BF16) is None and next_colder(Tier.DISK) is None
    assert next_colder(Tier.FP8) == Tier.INT4 and tier_distance(Tier.BF16, Tier.ARCHIVE) == 3
    ASHKVConfig()
    with pytest.raises(ValueError):
        ASHKVConfig(w_T=0.9)
    with pytest.raises(ValueError):
        ASHKVConfig(theta_low=0.8, theta_high=0.7)
    with pytest.raises(ValueError):
        ASHKVConfig(delta=-0.1)
    with pytest.raises(ValueError):
        ASHKVConfig(p_emergency=1.0)
    assert ASHKVConfig().as_dict()["theta_high"] == 0.72


def test_page_table_lifecycle():
    pt = PageTable(capacity=4)
    ids = [pt.add(i, 16 * i, 16 * i + 16, 100 + i, 7) for i in range(3)]
    assert ids == [0, 1, 2] and len(pt) == 3
    snap = pt.snapshot()
    assert snap.dtype == PAGE_DTYPE and snap["T"].tolist() == [1.0, 1.0, 1.0]
    snap["tier"][:] = 3
    assert pt.get_tier(0) == 0  # snapshot is a copy
    pt.pin(1)
    assert not pt.apply_tier_transition(1, Tier.FP8, 5)
    assert pt.apply_tier_transition(0, Tier.FP8, 5) and pt.get_tier(0) == 1
    pt.unpin(1)
    pt.unpin(1)
    assert pt.get_pin_count(1) == 0
    pt.remove(0)
    assert pt.find(0) == -1 and pt.get_tier(0) == -1 and pt.get_bf16_checksum(0) == 0 and len(pt) == 2
    assert pt.find(2) == 0  # last row swapped into the hole
    pt.update_score_inputs(np.array([1, 2, 99]), np.array([0.1, 0.2, 0.3], np.float32),
                           np.zeros(3, np.float32), np.zeros(3, np.float32), np.zeros(3, np.float32))
    assert pt.snapshot()["T"].tolist() == pytest.approx([0.2, 0.1])
    pt.add(9, 0, 16, 0, 0)
    pt.add(9, 0, 16, 0, 0)
    with pytest.raises(RuntimeError):
        pt.add(9, 0, 16, 0, 0)
    pt.touch(2, 42)
    assert pt.snapshot()["access_count"][pt.find(2)] == 1


def test_page_table_vectorised_ops():
    pt = PageTable(capacity=100)
    pids = pt.add_many(np.zeros(50, np.int32), np.arange(50, dtype=np.int32) * 16,
                       np.arange(50, dtype=np.int32) * 16 + 16, np.arange(50, dtype=np.uint64))
    assert pids.tolist() == list(range(50)) and pt.get_bf16_checksum(49) == 49
    pt.pin(3)
    ok = pt.apply_tier_transitions(np.array([2, 3, 4]), np.array([1, 1, 1], np.int8), np.array([7, 7, 7], np.uint64))
    assert ok.tolist() == [True, False, True] and pt.get_tier(3) == 0 and pt.get_tier(4) == 1


def test_protocols():
    assert isinstance(XorCodec(), Codec) and isinstance(MockAllocator(), Allocator)
    assert isinstance(SGLangShadowAllocator(10), Allocator)


# ------------------------------------------------------------------ migrate ladder
def run_migrate(codec=None, alloc=None, target=Tier.FP8, pin=False, lookup=None, breakers=None):
    alloc = alloc or MockAllocator()
    pt, pid, handles = setup_page(alloc)
    if isinstance(alloc, FaultyAllocator):
        alloc.armed = True
    if pin:
        pt.pin(pid)
    table = {} if codec is None else {(0, 1): codec, (1, 0): codec}
    return migrate(pid, target, pt, alloc, table, lookup or handles.__getitem__, lambda p: 256, breakers), pt, pid


def test_migrate_ok_commits_and_frees_source():
    alloc = MockAllocator()
    res, pt, pid = run_migrate(XorCodec(), alloc)
    assert res.status == MigrationStatus.OK and res.error == "" and pt.get_tier(pid) == 1
    assert res.from_tier == Tier.BF16 and res.to_tier == Tier.FP8 and res.duration_us >= 0
    assert alloc.num_allocations == 1  # target kept, source freed


@pytest.mark.parametrize("kwargs,status,error", [
    (dict(pin=True), MigrationStatus.SKIPPED, "pinned"),
    (dict(target=Tier.BF16), MigrationStatus.SKIPPED, "already at target"),
    (dict(codec=None), MigrationStatus.SKIPPED, "no codec"),
    (dict(lookup=lambda p: -1), MigrationStatus.FAILURE, "no handle"),
    (dict(lookup=lambda p: 1 / 0), MigrationStatus.FAILURE, "no handle"),
    (dict(alloc=FaultyAllocator("read")), MigrationStatus.FAILURE, "read failed"),
    (dict(codec=XorCodec(fail="encode")), MigrationStatus.FAILURE, "encode: injected encode failure"),
    (dict(alloc=FaultyAllocator("alloc")), MigrationStatus.FAILURE, "alloc failed"),
    (dict(codec=XorCodec(fail="decode")), MigrationStatus.FAILURE, "verify decode: injected decode failure"),
    (dict(codec=XorCodec(fail="checksum")), MigrationStatus.FAILURE, "verify checksum: injected checksum failure"),
    (dict(codec=XorCodec(corrupt=True)), MigrationStatus.CORRUPT, "checksum mismatch"),
])
def test_migrate_fault_ladder(kwargs, status, error):
    kwargs.setdefault("codec", XorCodec())
    res, pt, pid = run_migrate(**kwargs)
    assert isinstance(res, MigrationResult)
    assert res.status == status and res.error == error
    if status != MigrationStatus.OK:
        assert pt.get_tier(pid) in (0, -1)


def test_migrate_write_failure_frees_target():
    class WriteFailsOnce(MockAllocator):
        def __init__(self):
            super().__init__()
            self.n = 0

        def write(self, h, d):
            self.n += 1
            if self.n == 2:
                raise RuntimeError("write")
            super().write(h, d)

    alloc = WriteFailsOnce()
    res, pt, pid = run_migrate(XorCodec(), alloc)
    assert res.status == MigrationStatus.FAILURE and res.error == "write failed"
    assert alloc.num_allocations == 1


def test_migrate_missing_page_and_breaker():
    pt = PageTable(capacity=4)
    res = migrate(5, Tier.FP8, pt, MockAllocator(), {}, lambda p: 1, lambda p: 1)
    assert res.status == MigrationStatus.SKIPPED and res.error == "page not found"
    reg = CircuitBreakerRegistry()
    for _ in range(5):
        res, _, _ = run_migrate(XorCodec(fail="encode"), breakers=reg)
    assert not reg.is_codec_available("BF16_to_FP8")
    res, _, _ = run_migrate(XorCodec(), breakers=reg)
    assert res.status == MigrationStatus.SKIPPED and res.error == "breaker tripped"


def test_migrate_pin_race_rolls_back():
    alloc = MockAllocator()
    pt, pid, handles = setup_page(alloc)

    class PinningCodec(XorCodec):
        def checksum(self, b):
            pt.pin(pid)  # someone pins between snapshot and commit
            return super().checksum(b)

    res = migrate(pid, Tier.FP8, pt, alloc, {(0, 1): PinningCodec()}, handles.__getitem__, lambda p: 256)
    assert res.status == MigrationStatus.SKIPPED and res.error == "commit rejected (pin race)"
    assert alloc.num_allocations == 1  # only the source remains


# ------------------------------------------------------------------ registry / breaker / tables
def test_registry_freeze_and_duplicates():
    r = CodecRegistry()
    r.register("a", XorCodec())
    with pytest.raises(ValueError):
        r.register("a", XorCodec())
    r.freeze()
    with pytest.raises(RuntimeError):
        r.register("b", XorCodec())
    assert r.get("a") is not None and r.get("zzz") is None and r.names == ("a",) and r.frozen


def test_default_registry_has_the_reference_codec_names():
    """ashkv/codecs/__init__.py:26-32 of the reference registers these six names."""
    from ashkv.codecs import (BF16Codec, DitheredINT2Codec, DitheredNBitCodec, FP8Codec, INT4Codec,
                              INT8Codec)
    from ashkv.compiler.registry import codec_registry
    expect = {"bf16": BF16Codec, "int8_default": INT8Codec, "int4_default": INT4Codec,
              "int2_dithered": DitheredINT2Codec, "nbit_dithered": DitheredNBitCodec, "fp8_default": FP8Codec}
    for name, cls in expect.items():
        assert isinstance(codec_registry.get(name), cls), name
    # empty inputs never touch the device
    assert FP8Codec().encode(b"") == b"" and FP8Codec().decode(b"") == b""
    assert INT4Codec().encode(b"") == b"\0\0\0\0" and INT4Codec().decode(b"\0\0\0\0") == b""
    assert INT4Codec().decode(bytes(8)) == b""


def test_circuit_breaker_trip_and_cooldown():
    b = CircuitBreaker(threshold=3, window_seconds=60, cooldown_seconds=0.05)
    for _ in range(2):
        b.record_failure()
    assert not b.is_tripped and b.failure_count == 2
    b.record_failure()
    assert b.is_tripped
    b.record_success()
    assert b.is_tripped
    time.sleep(0.06)
    assert not b.is_tripped and b.failure_count == 0


def test_controller_tables_match_oracle():
    for keys in ([(0, 1), (1, 0)], [(0, 1), (1, 0), (1, 2), (2, 1), (0, 2), (2, 0), (2, 3), (3, 2)], []):
        nc, nh = controller_tables(keys)
        onc, onh = oracle.controller_tables(keys)
        assert nc.tolist() == onc.tolist() and nh.tolist() == onh.tolist()


# ------------------------------------------------------------------ hooks bookkeeping (data path stubbed)
class CpuPool:
    def __init__(self, host):
        import torch
        self.head_num, self.head_dim, self.layer_num = 32, 128, 1
        if host:
            self.k_buffer = torch.zeros((2048, 1, 32, 128), dtype=torch.bfloat16)
            self.v_buffer = torch.zeros((2048, 1, 32, 128), dtype=torch.bfloat16)
        else:
            self.k_buffer = [torch.zeros((2048, 32, 128), dtype=torch.bfloat16)]
            self.v_buffer = [torch.zeros((2048, 32, 128), dtype=torch.bfloat16)]


def test_hooks_byte_math_and_debounce(tmp_path, monkeypatch):
    import torch
    monkeypatch.chdir(tmp_path)
    monkeypatch.setattr(SGLangHooks, "_demote", lambda self, *a, **k: None)  # data path stubbed out
    dev, host = CpuPool(False), CpuPool(True)
    hooks = SGLangHooks()
    stats_file = tmp_path / "stats" / "ashkv_stats.json"
    assert stats_file.exists()
    mtime = os.path.getmtime(stats_file)
    with patch("time.time", return_value=0.5):
        for _ in range(100):
            assert hooks.demote_hook(dev, host, torch.arange(1), torch.arange(1), "MHA")
    assert os.path.getmtime(stats_file) == mtime
    assert json.loads(stats_file.read_text())["tokens_compressed"] == 0
    assert hooks.stats["tokens_compressed"] == 100
    hooks.stats = dict(hooks.stats, tokens_compressed=0, bytes_saved=0)
    with patch("time.time", return_value=5.0):
        hooks.demote_hook(dev, host, torch.arange(1024), torch.arange(1024), "MHA")
    assert hooks.stats["tokens_compressed"] == 1024
    assert hooks.stats["bytes_saved"] == 1024 * 32 * 128 * 4 - 1024 * (32 * 128 + 64) * 2
    assert json.loads(stats_file.read_text())["tokens_compressed"] == 1024


def test_hooks_decline_without_gpu(tmp_path, monkeypatch):
    import torch
    monkeypatch.chdir(tmp_path)
    hooks = SGLangHooks()
    dev, host = CpuPool(False), CpuPool(True)
    assert hooks.demote_hook(dev, host, torch.arange(3), torch.arange(3), "MLA") is False
    assert hooks.demote_hook(dev, host, torch.arange(0), torch.arange(0), "MHA") is False
    with pytest.raises(RuntimeError):
        hooks.demote_hook(dev, host, torch.arange(3), torch.arange(3), "MHA")  # CPU device pool


# ------------------------------------------------------------------ patcher
def _fake_sglang(mha, mla):
    mod = types.ModuleType("sglang.srt.mem_cache.memory_pool_host")
    mod.MHATokenToKVPoolHost, mod.MLATokenToKVPoolHost = mha, mla
    return {"sglang": types.ModuleType("sglang"), "sglang.srt": types.ModuleType("sglang.srt"),
            "sglang.srt.mem_cache": types.ModuleType("sglang.srt.mem_cache"),
            "sglang.srt.mem_cache.memory_pool_host": mod}


def _host_class():
    class Host:
        def backup_from_device_all_layer(self, dp, hi, di, io):
            return "orig_backup"

        def load_to_device_per_layer(self, dp, hi, di, layer, io):
            return "orig_load"
    return Host


def test_patcher_idempotent_and_fallback(caplog):
    mha, mla = _host_class(), _host_class()
    with patch.dict(sys.modules, _fake_sglang(mha, mla)):
        hooks = MagicMock()
        hooks.demote_hook.return_value = False
        hooks.promote_hook.return_value = True
        patcher_mod.apply_hicache_patches(hooks)
        first = mha.backup_from_device_all_layer
        patcher_mod.apply_hicache_patches(hooks)
        assert mha.backup_from_device_all_layer is first and mha.ashkv_patched and mla.ashkv_patched
        h = mha()
        assert h.backup_from_device_all_layer("dp", "hi", "di", None) is None  # declined -> original ran
        hooks.demote_hook.assert_called_with(device_pool="dp", host_pool=h, host_indices="hi", device_indices="di",
                                             pool_type="MHA", io_backend=None)
        h.load_to_device_per_layer("dp", "hi", "di", 3, None)
        assert hooks.promote_hook.call_args.kwargs["layer_id"] == 3
        mla().backup_from_device_all_layer("dp", "hi", "di", None)
        assert hooks.demote_hook.call_args.kwargs["pool_type"] == "MLA"


def test_patcher_without_hooks_or_sglang(caplog):
    mha = _host_class()
    with patch.dict(sys.modules, _fake_sglang(mha, _host_class())):
        patcher_mod.apply_hicache_patches(None)
        assert not getattr(mha, "ashkv_patched", False)
        assert "called without hooks" in caplog.text
    with patch.dict(sys.modules, {"sglang": None, "sglang.srt.mem_cache.memory_pool_host": None}):
        with pytest.raises(RuntimeError):
            patcher_mod.apply_hicache_patches(MagicMock())


# ------------------------------------------------------------------ arena allocator bookkeeping (no device use)
def test_shadow_allocator_bookkeeping():
    a = SGLangShadowAllocator(max_bytes=10_000)
    h1, h2 = a.alloc(Tier.FP8, 1000), a.alloc(Tier.FP8, 3000)
    assert (h1, h2) == (1, 2) and a.allocated_bytes == 4000 and a.pressure() == pytest.approx(0.4)
    assert a.alloc(Tier.FP8, 7000) == -1 and a.alloc(Tier.FP8, 0) == -1
    a.free(h2)
    a.free(h2)
    assert a.allocated_bytes == 1000
    h3 = a.alloc(Tier.FP8, 2000)  # fresh space first
    assert a.pool[h3][0] == 4096
    b = SGLangShadowAllocator(max_bytes=4096)
    x, y = b.alloc(Tier.FP8, 3000), b.alloc(Tier.FP8, 1000)
    b.free(x)
    z = b.alloc(Tier.FP8, 2000)  # no exact size, no fresh space: best fit splits the freed range
    assert b.pool[z][0] == 0 and b.pool[y][0] == 3072
    w = b.alloc(Tier.FP8, 1000)  # the 1024-byte remainder of the split
    assert b.pool[w][0] == 2048
    assert SGLangShadowAllocator(0).get_utilization() == 0.0
