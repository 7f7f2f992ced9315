"""The SGLang auto-patch loaded at interpreter start-up (ashkv/adapters/sglang/sitecustomize.py).

A child interpreter gets the adapter directory on PYTHONPATH (as an SGLang
worker would), so Python's ``site`` module imports the auto-patch; the child
then imports a stand-in ``sglang.srt.mem_cache.memory_pool_host`` and must see
its host-pool classes patched by the background thread, without the start-up
itself being delayed.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]
ADAPTER = REPO / "ash-kv_b200" / "ashkv" / "adapters" / "sglang"

CHILD = r'''
import sys, time, types
t0 = time.time()
assert "sitecustomize" in sys.modules and sys.modules["sitecustomize"].__file__.endswith("adapters/sglang/sitecustomize.py")
class MHATokenToKVPoolHost:
    def backup_from_device_all_layer(self, *a, **k): return "native"
    def load_to_device_per_layer(self, *a, **k): return "native"
class MLATokenToKVPoolHost(MHATokenToKVPoolHost):
    pass
names = ["sglang", "sglang.srt", "sglang.srt.mem_cache", "sglang.srt.mem_cache.memory_pool_host"]
for n in names:
    sys.modules[n] = types.ModuleType(n)
m = sys.modules[names[-1]]
m.MHATokenToKVPoolHost, m.MLATokenToKVPoolHost = MHATokenToKVPoolHost, MLATokenToKVPoolHost
for _ in range(200):
    if getattr(MHATokenToKVPoolHost, "ashkv_patched", False):
        break
    time.sleep(0.05)
assert MHATokenToKVPoolHost.ashkv_patched
assert MHATokenToKVPoolHost.backup_from_device_all_layer.__name__ == "backup_from_device_all_layer"
print("patched after", round(time.time() - t0, 2))
'''


def _env(**extra):
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join([str(ADAPTER), str(REPO / "ash-kv_b200")])
    env["ASHKV_PATCH_DELAY_S"] = "0.05"
    env.update(extra)
    return env


def test_autopatch_applies_in_a_fresh_interpreter(tmp_path):
    r = subprocess.run([sys.executable, "-c", CHILD], cwd=tmp_path, env=_env(), capture_output=True, text=True,
                       timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "patched after" in r.stdout
    log = (tmp_path / "stats" / "ashkv_patch.log").read_text()
    assert "background thread started" in log and "patches applied" in log


def test_autopatch_can_be_disabled(tmp_path):
    code = "import sys; print('sitecustomize' in sys.modules)"
    r = subprocess.run([sys.executable, "-c", code], cwd=tmp_path, env=_env(ASHKV_DISABLE_PATCHES="1"),
                       capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    assert not (tmp_path / "stats" / "ashkv_patch.log").exists()
