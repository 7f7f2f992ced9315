"""Auto-patch SGLang's HiCache in every process that loads this file at start-up.

Same role as the reference's ``sitecustomize`` (ashkv/adapters/sglang/
sitecustomize.py:7-33): SGLang's tensor-parallel workers are separate
processes (spawned by SGLang or by Ray, which drops most environment
variables), so the hooks cannot be installed from the launching process.
Put this directory on ``PYTHONPATH``; Python's ``site`` module then imports
this file in every interpreter, which starts a daemon thread that waits until
``sglang.srt.mem_cache.memory_pool_host`` has been imported, waits a moment
for the module to finish initialising, and calls ``apply_hicache_patches``
with ``SGLangHooks(codec_name="int8_default")``.  Processes that never import
SGLang only carry an idle daemon thread.  Progress is appended to
``stats/ashkv_patch.log`` (relative to the working directory), as the
reference does.

Set ``ASHKV_DISABLE_PATCHES=1`` to skip the thread; ``ASHKV_PATCH_DELAY_S``
changes the settle delay after SGLang appears (default 2 seconds).
"""
from __future__ import annotations

import os
import sys
import threading
import time

_TARGET = "sglang.srt.mem_cache.memory_pool_host"
_LOG = os.path.join("stats", "ashkv_patch.log")


def _log(msg: str) -> None:
    try:
        os.makedirs("stats", exist_ok=True)
        with open(_LOG, "a") as f:
            f.write(f"[ASH-KV] {msg}\n")
    except OSError:
        pass


def _delayed_patch(poll_s: float = 0.5) -> None:
    _log(f"background thread started in process {os.getpid()}")
    while _TARGET not in sys.modules:
        time.sleep(poll_s)
    time.sleep(float(os.environ.get("ASHKV_PATCH_DELAY_S", "2.0")))
    try:
        from ashkv.adapters.sglang.hooks import SGLangHooks
        from ashkv.adapters.sglang.patcher import apply_hicache_patches
        apply_hicache_patches(SGLangHooks(codec_name="int8_default"))
        _log("patches applied")
    except Exception as e:  # noqa: BLE001 -- never break the host process
        _log(f"failed to auto-patch: {e}")


if os.environ.get("ASHKV_DISABLE_PATCHES") != "1":
    threading.Thread(target=_delayed_patch, name="ashkv-autopatch", daemon=True).start()
