"""Cold-path helpers: the codec registry and the controller's lookup tables."""
from __future__ import annotations

from .codec_resolver import CodecConfig, page_format, resolve_codecs, tier_formats
from .hardware_probe import HardwareProfile, probe_hardware
from .registry import CodecRegistry, codec_registry
from .runtime_builder import build_runtime, compile_controller, compile_score, controller_tables

__all__ = ["CodecRegistry", "codec_registry", "build_runtime", "compile_controller", "compile_score",
           "controller_tables", "CodecConfig", "resolve_codecs", "page_format", "tier_formats",
           "HardwareProfile", "probe_hardware"]
