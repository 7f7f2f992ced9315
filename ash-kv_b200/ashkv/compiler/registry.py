"""Codec registry: name -> codec instance, frozen after startup.

Same behaviour as ``CodecRegistry`` in ashkv/compiler/registry.py:18-65 of
the reference: duplicate names raise ValueError, registering after
``freeze()`` raises RuntimeError, ``get`` returns None for unknown names.
"""
from __future__ import annotations

from typing import Dict

from ..contracts.protocols import Codec


class CodecRegistry:
    __slots__ = ("_by_name", "_frozen")

    def __init__(self) -> None:
        self._by_name: Dict[str, Codec] = {}
        self._frozen = False

    def register(self, name: str, codec: Codec) -> None:
        if self._frozen:
            raise RuntimeError(f"CodecRegistry is frozen; cannot register '{name}'. "
                               f"All registrations must happen at startup.")
        if name in self._by_name:
            raise ValueError(f"Codec '{name}' already registered")
        self._by_name[name] = codec

    def get(self, name: str) -> Codec | None:
        return self._by_name.get(name)

    def freeze(self) -> None:
        self._frozen = True

    @property
    def frozen(self) -> bool:
        return self._frozen

    @property
    def names(self) -> tuple[str, ...]:
        return tuple(self._by_name)


codec_registry = CodecRegistry()
