"""Monkey-patch SGLang's HiCache host pools to route through SGLangHooks.

Same behaviour as ``apply_hicache_patches`` (ashkv/adapters/sglang/patcher.py:17-111
of the reference): without hooks it logs a warning and patches nothing; it
needs ``sglang.srt.mem_cache.memory_pool_host`` (RuntimeError otherwise); it is
idempotent (``ashkv_patched`` marker); a hook returning False falls back to
the original method.
"""
from __future__ import annotations

import logging
import threading

logger = logging.getLogger(__name__)

_HOOKS = None
_PATCH_LOCK = threading.Lock()


def _wrap(cls, pool_type: str) -> None:
    orig_backup = cls.backup_from_device_all_layer
    orig_load = cls.load_to_device_per_layer

    def backup_from_device_all_layer(self, device_pool, host_indices, device_indices, io_backend):
        if not _HOOKS.demote_hook(device_pool=device_pool, host_pool=self, host_indices=host_indices,
                                  device_indices=device_indices, pool_type=pool_type, io_backend=io_backend):
            orig_backup(self, device_pool, host_indices, device_indices, io_backend)

    def load_to_device_per_layer(self, device_pool, host_indices, device_indices, layer_id, io_backend):
        if not _HOOKS.promote_hook(device_pool=device_pool, host_pool=self, host_indices=host_indices,
                                   device_indices=device_indices, layer_id=layer_id, pool_type=pool_type,
                                   io_backend=io_backend):
            orig_load(self, device_pool, host_indices, device_indices, layer_id, io_backend)

    cls.backup_from_device_all_layer = backup_from_device_all_layer
    cls.load_to_device_per_layer = load_to_device_per_layer
    cls.ashkv_patched = True


def apply_hicache_patches(hooks=None) -> None:
    global _HOOKS
    _HOOKS = hooks
    if _HOOKS is None:
        logger.warning("apply_hicache_patches called without hooks; interception will be disabled.")
        return
    try:
        from sglang.srt.mem_cache.memory_pool_host import MHATokenToKVPoolHost, MLATokenToKVPoolHost
    except ImportError as e:
        logger.error("Failed to import SGLang HostKVCache. ASH-KV requires SGLang >= 0.5.x for HiCache.")
        raise RuntimeError(f"Incompatible SGLang version or missing dependency: {e}")
    with _PATCH_LOCK:
        if getattr(MHATokenToKVPoolHost, "ashkv_patched", False):
            return
        _wrap(MHATokenToKVPoolHost, "MHA")
        _wrap(MLATokenToKVPoolHost, "MLA")
    logger.info("ASH-KV successfully patched SGLang HiCache (HostKVCache).")
