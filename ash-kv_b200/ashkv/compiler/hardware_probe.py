"""Hardware profile for codec resolution (cold path).

Same fields and rules as ``probe_hardware`` (ashkv/compiler/hardware_probe.py:
12-101 of the reference): NVIDIA compute capability >= 9.0 has native FP8,
>= 7.5 INT8, >= 8.0 BF16; an AMD Instinct MI300-class part has FP8; without a
GPU the profile has no acceleration.  One difference: the reference reads
``props.total_mem``, an attribute torch's device properties do not have, so on
a real GPU its probe falls into its CPU-profile fallback (and its resolver then
picks ``int8_default``).  This probe reads ``total_memory`` and reports the
device as it is; pass ``CodecConfig(bf16_to_compressed="int8_default")`` for the
reference's effective choice.  No warm-up is needed (no JIT compiler).
"""
from __future__ import annotations

import logging
from dataclasses import dataclass

logger = logging.getLogger("ashkv.compiler.hardware_probe")


@dataclass(frozen=True, slots=True)
class HardwareProfile:
    gpu_name: str
    compute_capability: tuple[int, int]
    vram_bytes: int
    has_fp8_native: bool
    has_int8_native: bool
    has_bf16_native: bool
    is_amd: bool


def cpu_profile() -> HardwareProfile:
    return HardwareProfile("CPU", (0, 0), 0, False, False, False, False)


def profile_for(name: str, cc: tuple[int, int], vram_bytes: int) -> HardwareProfile:
    is_amd = "AMD" in name.upper() or "Instinct" in name.upper()
    if is_amd:
        has_fp8 = any(m in name for m in ("MI300", "MI325", "MI350"))
        has_int8 = has_bf16 = True
    else:
        has_fp8, has_int8, has_bf16 = cc >= (9, 0), cc >= (7, 5), cc >= (8, 0)
    return HardwareProfile(name, cc, vram_bytes, has_fp8, has_int8, has_bf16, is_amd)


def probe_hardware(device_id: int = 0) -> HardwareProfile:
    """Profile of CUDA device ``device_id`` (the CPU profile when there is none). Never raises."""
    try:
        import torch
        if not torch.cuda.is_available():
            return cpu_profile()
        props = torch.cuda.get_device_properties(device_id)
        return profile_for(props.name, (props.major, props.minor), int(props.total_memory))
    except Exception as e:  # noqa: BLE001 -- the probe never raises, like the reference's
        logger.warning("hardware probe failed: %s; using the CPU profile", e)
        return cpu_profile()
