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


def assert_int8_codes(got, want, tie) -> int:
    """INT8 codes against the oracle: equal, except one apart at tie-zone elements.

    The reference's Triton kernel (and this library, which reproduces it) divides
    with the GPU's approximate ``div.full.f32``; the oracle divides exactly and
    marks the elements whose exact quotient lies next to a half-integer, the only
    place the two can round to neighbouring codes.  Returns how many codes differ
    (all at ties).  Exact agreement with the reference itself is tested against
    the B200 fixtures in ``tests/test_gpu_reference_fixtures.py``."""
    import oracle
    ok, n = oracle.int8_codes_agree(got, want, tie)
    assert ok, "INT8 codes differ from the oracle outside the tie zone (or by more than one)"
    return n


def assert_int8_roundtrip(got_u16, src_u16, row_len: int, scale_fp16: bool = True) -> None:
    """bf16 rows decoded from INT8 codes of ``src_u16`` rows: equal to the oracle's
    decode of its own codes, or, at tie-zone elements, to the decode of the
    neighbouring code."""
    import numpy as np
    import oracle
    src = np.ascontiguousarray(src_u16, dtype=np.uint16).reshape(-1, row_len)
    codes, scales, tie = oracle.int8_encode(src, row_len, scale_fp16=scale_fp16, with_ties=True)
    got = np.asarray(got_u16, dtype=np.uint16).reshape(src.shape)
    ok = got == oracle.int8_decode(codes, scales, scale_fp16=scale_fp16)
    for step in (-1, 1):
        alt = np.clip(codes.astype(np.int16) + step, -128, 127).astype(np.int8)
        ok |= tie & (got == oracle.int8_decode(alt, scales, scale_fp16=scale_fp16))
    assert ok.all(), f"{int((~ok).sum())} decoded values differ from the oracle outside the tie zone"
