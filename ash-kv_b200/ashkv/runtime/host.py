"""Host-side placement for pinned transfers: keep a rank's host threads and its
pinned buffers on the CPU socket its GPU is attached to.

Pinned (page-locked) host memory is placed on the NUMA node of the thread that
first touches it, and every host<->device copy of a rank crosses that node's
memory controllers.  When the eight ranks of a box run wherever the scheduler
puts them, half of their DMA traffic crosses the socket interconnect and the
ranks' copies contend there.  ``bind_to_device(device)`` restricts the calling
process to the CPUs local to the GPU (the PCI device's ``local_cpulist`` in
sysfs) so that pinned buffers allocated afterwards live on that GPU's node.
It changes only this process's CPU affinity; nothing of the GPU is touched.
"""
from __future__ import annotations

import os
from pathlib import Path
from typing import Optional

import torch


def _parse_cpulist(text: str) -> set[int]:
    cpus: set[int] = set()
    for part in text.strip().split(","):
        if not part:
            continue
        if "-" in part:
            a, b = part.split("-")
            cpus.update(range(int(a), int(b) + 1))
        else:
            cpus.add(int(part))
    return cpus


def pci_bus_id(device: torch.device) -> Optional[str]:
    """The device's PCI address as sysfs names it (``dddd:bb:dd.0``), or None."""
    try:
        p = torch.cuda.get_device_properties(device)
        return f"{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
    except Exception:  # noqa: BLE001 -- no CUDA, or properties without PCI fields
        return None


def device_local_cpus(device: torch.device, sysfs: Path = Path("/sys/bus/pci/devices")) -> Optional[set[int]]:
    """CPUs local to the GPU (sysfs ``local_cpulist`` of its PCI device), or None if unknown."""
    bus = pci_bus_id(device)
    if bus is None:
        return None
    f = sysfs / bus / "local_cpulist"
    try:
        cpus = _parse_cpulist(f.read_text())
    except (OSError, ValueError):
        return None
    return cpus or None


def bind_to_device(device: torch.device) -> Optional[dict]:
    """Restrict this process to the CPUs local to ``device`` (intersected with the CPUs it
    may use now).  Returns what was done, or None when the locality is unknown or the
    process may not run on any local CPU (the affinity is then left unchanged)."""
    local = device_local_cpus(device)
    if not local or not hasattr(os, "sched_setaffinity"):
        return None
    allowed = os.sched_getaffinity(0)
    cpus = local & allowed
    if not cpus:
        return None
    if cpus != allowed:
        os.sched_setaffinity(0, cpus)
    return {"pci_bus_id": pci_bus_id(device), "cpus": len(cpus), "of": len(allowed)}
