"""The C-ABI library: loads without a GPU, exports every declared symbol,
and validates arguments on the host before touching the device."""
from __future__ import annotations

import ctypes
import re

from conftest import REPO

from ashkv import _native

HEADER = (REPO / "include" / "ashkv.h").read_text()
DECLARED = re.findall(r"^ASHKV_API\s+[\w\s\*]+?\b(ashkv_\w+)\s*\(", HEADER, flags=re.M)


def test_header_declares_entry_points():
    assert len(DECLARED) >= 15
    assert "ashkv_nbit_encode" in DECLARED and "ashkv_policy_step" in DECLARED


def test_library_exports_every_declared_symbol():
    lib = _native.lib()
    for name in DECLARED:
        assert hasattr(lib, name), name


def test_binding_covers_every_declared_symbol():
    assert set(DECLARED) <= set(_native.SIGNATURES), set(DECLARED) - set(_native.SIGNATURES)


def test_version_and_status_strings():
    lib = _native.lib()
    assert lib.ashkv_version() >= 100
    assert _native.status_string(0) == "ok"
    assert _native.status_string(_native.BAD_ARGUMENT) == "bad argument"
    assert _native.status_string(_native.OUTLIER_OVERFLOW) == "outlier capacity overflow"
    assert _native.status_string(99) == "unknown status"


def test_host_side_argument_validation_without_gpu():
    lib = _native.lib()
    null = None
    # bits must be 2, 4 or 8
    assert lib.ashkv_nbit_encode(null, 4, 3, 3.0, 0, null, 0, 0, null, null, null, null, 0, null, null) == 1
    # empty inputs are a no-op
    assert lib.ashkv_nbit_encode(null, 0, 4, 3.0, 1, null, 0, 0, null, null, null, null, 0, null, null) == 0
    # Philox counter offset must be a multiple of 8
    assert lib.ashkv_nbit_encode(ctypes.c_void_p(16), 4, 4, 3.0, 1, null, 0, 3, ctypes.c_void_p(16),
                                 ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.c_void_p(16), 8,
                                 ctypes.c_void_p(16), null) == 1
    # misaligned source pointer
    assert lib.ashkv_nbit_encode(ctypes.c_void_p(18), 4, 4, 3.0, 1, null, 0, 0, ctypes.c_void_p(16),
                                 ctypes.c_void_p(16), ctypes.c_void_p(16), ctypes.c_void_p(16), 8,
                                 ctypes.c_void_p(16), null) == 1
    assert lib.ashkv_int8_encode_rows(null, 0, -1, 128, 128, null, null, 128, null, 0, 1, 2, 0, null) == 1
    assert lib.ashkv_int8_encode_rows(null, 7, 4, 128, 128, null, null, 128, null, 0, 1, 2, 0, null) == 1
    assert lib.ashkv_int8_decode_rows(null, 128, null, 0, 0, 2, 4, 128, null, 0, 128, null, null) == 1
    assert lib.ashkv_xxh64_items(null, 0, 32, 32, 0, null, null) == 0
    assert lib.ashkv_xxh64_items(null, 2, 64, 32, 0, ctypes.c_void_p(8), null) == 1  # stride < size
    assert lib.ashkv_score(null, null, null, null, 0, 0.7, 0.1, 0.1, 0.1, null, null) == 0
    tbl = (ctypes.c_int8 * 6)(1, 2, 3, 4, 5, 5)
    assert lib.ashkv_desired_tiers(null, null, -1, 0.5, 0.72, 0.33, 0.04, 0.95, ctypes.addressof(tbl),
                                   ctypes.addressof(tbl), null, null) == 1
    assert lib.ashkv_policy_scratch_ints(1 << 20) == 2 * 1024 + 2
