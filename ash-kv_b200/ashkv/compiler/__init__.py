"""Cold-path helpers: the codec registry and the controller's lookup tables."""
from __future__ import annotations

from .registry import CodecRegistry, codec_registry
from .runtime_builder import build_runtime, compile_controller, compile_score, controller_tables

__all__ = ["CodecRegistry", "codec_registry", "build_runtime", "compile_controller", "compile_score",
           "controller_tables"]
