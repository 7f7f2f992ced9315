"""Host placement helper (ashkv/runtime/host.py) against a fake sysfs tree."""
from __future__ import annotations

import os

import pytest
import torch

from ashkv.runtime import host


def test_parse_cpulist():
    assert host._parse_cpulist("0-3,8,10-11\n") == {0, 1, 2, 3, 8, 10, 11}
    assert host._parse_cpulist("") == set()


def test_local_cpus_from_sysfs(tmp_path, monkeypatch):
    d = tmp_path / "0000:1b:00.0"
    d.mkdir()
    (d / "local_cpulist").write_text("0-3,6\n")
    monkeypatch.setattr(host, "pci_bus_id", lambda dev: "0000:1b:00.0")
    assert host.device_local_cpus(torch.device("cuda", 0), sysfs=tmp_path) == {0, 1, 2, 3, 6}
    monkeypatch.setattr(host, "pci_bus_id", lambda dev: "0000:99:00.0")
    assert host.device_local_cpus(torch.device("cuda", 0), sysfs=tmp_path) is None


@pytest.mark.skipif(not hasattr(os, "sched_setaffinity"), reason="no CPU affinity on this platform")
def test_bind_restricts_to_local_cpus_and_back(monkeypatch):
    before = os.sched_getaffinity(0)
    one = min(before)
    monkeypatch.setattr(host, "device_local_cpus", lambda dev: {one, 10 ** 6})
    monkeypatch.setattr(host, "pci_bus_id", lambda dev: "0000:1b:00.0")
    try:
        r = host.bind_to_device(torch.device("cuda", 0))
        assert r == {"pci_bus_id": "0000:1b:00.0", "cpus": 1, "of": len(before)}
        assert os.sched_getaffinity(0) == {one}
        # no local CPU the process may use: affinity left as it is
        monkeypatch.setattr(host, "device_local_cpus", lambda dev: {10 ** 6})
        assert host.bind_to_device(torch.device("cuda", 0)) is None
        assert os.sched_getaffinity(0) == {one}
    finally:
        os.sched_setaffinity(0, before)
