"""Shared pytest setup: import paths, the ``gpu`` marker, library build."""
from __future__ import annotations

import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
for p in (str(REPO), str(REPO / "ash-kv_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def _have_gpu() -> bool:
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@pytest.fixture(scope="session", autouse=True)
def _built_library():
    """Make sure libashkv_cuda.so matches the sources (nvcc cross-compiles on CPU hosts)."""
    from ashkv import _build
    if _build.needs_build():
        _build.build_library()
    yield


@pytest.fixture(scope="session")
def cuda():
    if not _have_gpu():
        pytest.skip("no CUDA device")
    import torch
    torch.cuda.init()
    return torch.device("cuda", 0)


GOLDEN = REPO / "tests" / "golden"
