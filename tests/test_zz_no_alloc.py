"""The allocation-free policy step (ashkv_policy_step_noalloc).

Callers that cannot allocate device memory while planning a step (an engine
that reserved nearly all HBM for its KV pool, a plain C/FFI caller without a
caching allocator) use this entry point: it takes no scratch buffer and keeps
its per-block counts in a static device array inside the library.  The test
calls it through the C ABI twice in a row and compares every output with the
regular ashkv_policy_step, which gets caller-provided scratch.  This file
sorts last so a run that stops at the first failure has run all other tests.
"""
from __future__ import annotations

import pytest
import torch

from ashkv import _native
from ashkv.compiler import controller_tables

pytestmark = pytest.mark.gpu


def _inputs(cuda, n, seed):
    g = torch.Generator(device=cuda).manual_seed(seed)
    feats = [torch.rand(n, generator=g, device=cuda) for _ in range(4)]
    cur = torch.randint(0, 4, (n,), generator=g, device=cuda, dtype=torch.int8)
    return feats, cur


def _outputs(cuda, n):
    return (torch.empty(n, device=cuda), torch.empty(n, dtype=torch.int8, device=cuda),
            torch.empty(n, dtype=torch.int32, device=cuda), torch.empty(n, dtype=torch.int32, device=cuda),
            torch.zeros(2, dtype=torch.int32, device=cuda))


def test_noalloc_matches_scratch_version_twice(cuda):
    nc, nh = controller_tables([(0, 1), (1, 0), (1, 2), (2, 1), (0, 2), (2, 0), (2, 3), (3, 2)])
    for call, (n, pressure, seed) in enumerate([(1 << 20, 0.97, 1), (300_001, 0.9, 2)]):
        (T, S, N, P), cur = _inputs(cuda, n, seed)
        R0, t0, d0, p0, c0 = _outputs(cuda, n)
        scratch = torch.empty(_native.policy_scratch_ints(n), dtype=torch.int32, device=cuda)
        _native.policy_step(T, S, N, P, cur, (0.7, 0.1, 0.1, 0.1), pressure, 0.72, 0.33, 0.04, 0.95, nc, nh,
                            R0, t0, d0, p0, c0, scratch)
        R1, t1, d1, p1, c1 = _outputs(cuda, n)
        _native.policy_step_noalloc(T, S, N, P, cur, (0.7, 0.1, 0.1, 0.1), pressure, 0.72, 0.33, 0.04, 0.95, nc,
                                    nh, R1, t1, d1, p1, c1)
        torch.cuda.synchronize()
        assert torch.equal(R0, R1) and torch.equal(t0, t1) and torch.equal(c0, c1), call
        nd, npro = c0.tolist()
        assert nd > 0 and torch.equal(d0[:nd], d1[:nd]) and torch.equal(p0[:npro], p1[:npro]), call


def test_noalloc_rejects_tables_beyond_its_static_scratch(cuda):
    n = _native.POLICY_NOALLOC_MAX_PAGES + 1
    nc, nh = controller_tables([(0, 1), (1, 0)])
    one = torch.zeros(1, device=cuda)
    c = torch.zeros(1, dtype=torch.int8, device=cuda)
    i32 = torch.zeros(1, dtype=torch.int32, device=cuda)
    lib = _native.lib()
    a, b = _native._table(nc), _native._table(nh)
    rc = lib.ashkv_policy_step_noalloc(one.data_ptr(), one.data_ptr(), one.data_ptr(), one.data_ptr(), c.data_ptr(),
                                       n, 0.7, 0.1, 0.1, 0.1, 0.5, 0.72, 0.33, 0.04, 0.95, _native._addr(a),
                                       _native._addr(b), None, c.data_ptr(), i32.data_ptr(), i32.data_ptr(),
                                       i32.data_ptr(), None)
    assert rc == _native.BAD_ARGUMENT
    assert "static scratch" in lib.ashkv_last_error().decode()
