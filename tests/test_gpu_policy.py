"""GPU parity: page-table policy kernels and per-page XXH64 against the oracle/reference."""
from __future__ import annotations

import numpy as np
import pytest
import torch
import xxhash

import oracle
from conftest import GOLDEN

from ashkv import _native
from ashkv.codecs import checksum_pages
from ashkv.compiler import controller_tables
from ashkv.runtime import desired_tiers, score_vectorized

pytestmark = pytest.mark.gpu

POLICY = np.load(GOLDEN / "policy.npz")


def test_score_and_tiers_match_reference_golden(cuda):
    z = POLICY
    R = score_vectorized(z["policy_T"], z["policy_S"], z["policy_N"], z["policy_P"], 0.7, 0.1, 0.1, 0.1)
    assert isinstance(R, np.ndarray) and R.dtype == np.float32
    assert np.array_equal(R, z["policy_R"], equal_nan=True)
    nc, nh = controller_tables([tuple(k) for k in z["policy_codec_keys"]])
    for i, p in enumerate(z["policy_pressures"]):
        t = desired_tiers(R, z["policy_cur"], float(p), 0.72, 0.33, 0.04, 0.95, nc, nh)
        assert t.dtype == np.int8
        assert np.array_equal(t, z[f"policy_target_{i}"]), p
    R2 = score_vectorized(z["policy_T"], z["policy_S"], z["policy_N"], z["policy_P"], 0.55, 0.15, 0.2, 0.1)
    assert np.array_equal(R2, z["policy_R2"], equal_nan=True)
    t2 = desired_tiers(R2, z["policy_cur"], 0.963, 0.61, 0.29, 0.03, 0.9, nc, nh)
    assert np.array_equal(t2, z["policy_target_alt"])


def test_reference_runtime_examples(cuda):
    T = np.array([1.0, 0.5, 0.0], dtype=np.float32)
    S = np.array([0.0, 0.5, 1.0], dtype=np.float32)
    Z = np.zeros(3, dtype=np.float32)
    assert np.allclose(score_vectorized(T, S, Z, Z, 0.7, 0.1, 0.1, 0.1), [0.7, 0.4, 0.1], atol=1e-6)
    assert len(score_vectorized(T, S[:1], Z, Z, 0.7, 0.1, 0.1, 0.1)) == 0
    assert len(score_vectorized(T[:0], S[:0], Z[:0], Z[:0], 0.7, 0.1, 0.1, 0.1)) == 0
    nc, nh = controller_tables([(0, 1), (1, 0), (1, 2), (2, 1)])
    cur = np.array([1, 2, 0, 0], dtype=np.int8)
    R = np.array([0.9, 0.9, 0.1, 0.5], dtype=np.float32)
    t = desired_tiers(R, cur, 0.5, 0.72, 0.33, 0.04, 0.95, nc, nh)
    assert t.tolist() == [0, 1, 1, 0]
    empty = desired_tiers(R[:0], cur[:0], 0.5, 0.72, 0.33, 0.04, 0.95, nc, nh)
    assert len(empty) == 0
    mism = desired_tiers(R[:2], cur, 0.5, 0.72, 0.33, 0.04, 0.95, nc, nh)
    assert mism.tolist() == cur.tolist()


def test_device_tensors_stay_on_device(cuda):
    n = 1000
    g = torch.Generator(device=cuda).manual_seed(1)
    T, S, N, P = (torch.rand(n, generator=g, device=cuda) for _ in range(4))
    R = score_vectorized(T, S, N, P, 0.7, 0.1, 0.1, 0.1)
    assert R.is_cuda
    want = oracle.score(*(a.cpu().numpy() for a in (T, S, N, P)), 0.7, 0.1, 0.1, 0.1)
    assert np.array_equal(R.cpu().numpy(), want)
    cur = torch.randint(0, 4, (n,), device=cuda, dtype=torch.int8)
    nc, nh = controller_tables([(0, 1), (1, 0), (1, 2), (2, 1), (2, 3), (3, 2)])
    t = desired_tiers(R, cur, 0.97, 0.72, 0.33, 0.04, 0.95, nc, nh)
    assert t.is_cuda and t.dtype == torch.int8
    assert np.array_equal(t.cpu().numpy(), oracle.desired_tiers(want, cur.cpu().numpy(), 0.97, 0.72, 0.33, 0.04,
                                                                0.95, nc, nh))


@pytest.mark.parametrize("pressure", [0.5, 0.7, 0.9, 0.95, 0.96, 0.97])
def test_policy_step_lists_config5(cuda, pressure):
    """The mixed-tier plan at scale: 1,048,576 pages, tiers uniform in {0..3}, pressure sweep."""
    n = 1 << 20
    g = torch.Generator(device=cuda).manual_seed(int(pressure * 100))
    T, S, N, P = (torch.rand(n, generator=g, device=cuda) for _ in range(4))
    cur = torch.randint(0, 4, (n,), generator=g, device=cuda, dtype=torch.int8)
    nc, nh = controller_tables([(0, 1), (1, 0), (1, 2), (2, 1), (0, 2), (2, 0), (2, 3), (3, 2)])
    R = torch.empty(n, device=cuda)
    target = torch.empty(n, dtype=torch.int8, device=cuda)
    dl = torch.empty(n, dtype=torch.int32, device=cuda)
    pl = torch.empty(n, dtype=torch.int32, device=cuda)
    counts = torch.empty(2, dtype=torch.int32, device=cuda)
    scratch = torch.empty(_native.policy_scratch_ints(n), dtype=torch.int32, device=cuda)
    _native.policy_step(T, S, N, P, cur, (0.7, 0.1, 0.1, 0.1), pressure, 0.72, 0.33, 0.04, 0.95, nc, nh, R, target,
                        dl, pl, counts, scratch)
    Rn = oracle.score(*(a.cpu().numpy() for a in (T, S, N, P)), 0.7, 0.1, 0.1, 0.1)
    cn = cur.cpu().numpy()
    tn = oracle.desired_tiers(Rn, cn, pressure, 0.72, 0.33, 0.04, 0.95, nc, nh)
    assert np.array_equal(R.cpu().numpy(), Rn)
    assert np.array_equal(target.cpu().numpy(), tn)
    nd, npro = counts.cpu().tolist()
    assert np.array_equal(dl[:nd].cpu().numpy(), np.nonzero(tn > cn)[0])
    assert np.array_equal(pl[:npro].cpu().numpy(), np.nonzero(tn < cn)[0])


@pytest.mark.parametrize("pressure", [0.5, 0.9, 0.95, 0.96, 0.97, 0.999, float("nan")])
def test_policy_step_device_pressure_matches_host(cuda, pressure):
    """The pressure read on the device (fp32, as after the ranks' all-reduce) gives the
    lists the host path gives for the same fp32 value, with caller scratch or the
    library's static scratch."""
    n = 300_000
    g = torch.Generator(device=cuda).manual_seed(7)
    T, S, N, P = (torch.rand(n, generator=g, device=cuda) for _ in range(4))
    cur = torch.randint(0, 4, (n,), generator=g, device=cuda, dtype=torch.int8)
    nc, nh = controller_tables([(0, 1), (1, 0), (1, 2), (2, 1), (0, 2), (2, 0), (2, 3), (3, 2)])
    p32 = torch.tensor([pressure], dtype=torch.float32, device=cuda)
    outs = []
    for mode in ("host", "device", "device_static"):
        R = torch.empty(n, device=cuda)
        target = torch.empty(n, dtype=torch.int8, device=cuda)
        dl = torch.full((n,), -1, dtype=torch.int32, device=cuda)
        pl = torch.full((n,), -1, dtype=torch.int32, device=cuda)
        counts = torch.empty(2, dtype=torch.int32, device=cuda)
        scratch = torch.empty(_native.policy_scratch_ints(n), dtype=torch.int32, device=cuda)
        if mode == "host":
            _native.policy_step(T, S, N, P, cur, (0.7, 0.1, 0.1, 0.1), float(p32.item()), 0.72, 0.33, 0.04, 0.95,
                                nc, nh, R, target, dl, pl, counts, scratch)
        elif mode == "device":
            _native.policy_step(T, S, N, P, cur, (0.7, 0.1, 0.1, 0.1), p32, 0.72, 0.33, 0.04, 0.95,
                                nc, nh, R, target, dl, pl, counts, scratch)
        else:
            ncb = np.ascontiguousarray(nc, dtype=np.int8)
            nhb = np.ascontiguousarray(nh, dtype=np.int8)
            _native.check(_native.lib().ashkv_policy_step_device_pressure(
                T.data_ptr(), S.data_ptr(), N.data_ptr(), P.data_ptr(), cur.data_ptr(), n, 0.7, 0.1, 0.1, 0.1,
                p32.data_ptr(), 0.72, 0.33, 0.04, 0.95, ncb.ctypes.data, nhb.ctypes.data, R.data_ptr(),
                target.data_ptr(), dl.data_ptr(), pl.data_ptr(), counts.data_ptr(), None,
                _native.stream_handle(cuda)), "policy_step_device_pressure")
        torch.cuda.synchronize()
        outs.append([t.cpu().numpy() for t in (R, target, dl, pl, counts)])
    Rn = oracle.score(*(a.cpu().numpy() for a in (T, S, N, P)), 0.7, 0.1, 0.1, 0.1)
    tn = oracle.desired_tiers(Rn, cur.cpu().numpy(), float(np.float32(pressure)), 0.72, 0.33, 0.04, 0.95, nc, nh)
    for o in outs:
        assert np.array_equal(o[1], tn)
        for a, b in zip(o, outs[0]):
            assert np.array_equal(a, b)


@pytest.mark.parametrize("item_bytes,stride", [(32768, 32768), (32768, 33024), (1, 8), (31, 40), (100, 100),
                                               (77, 77), (4096 + 24, 4096 + 24), (4096 + 24, 4096 + 32),
                                               (1024, 1024), (1040, 1040), (5000, 5008), (65536 + 7, 65536 + 16)])
def test_xxh64_items_match_xxhash(cuda, item_bytes, stride):
    n = 64
    rng = np.random.default_rng(item_bytes)
    buf = rng.integers(0, 256, n * stride + 16, dtype=np.uint8)
    d = torch.from_numpy(buf).to(cuda)
    out = torch.empty(n, dtype=torch.int64, device=cuda)
    for seed in (0, 12345):
        _native.xxh64_items(d, n, item_bytes, stride, out, seed)
        got = out.cpu().numpy().view(np.uint64)
        want = [xxhash.xxh64(buf[i * stride:i * stride + item_bytes].tobytes(), seed=seed).intdigest()
                for i in range(n)]
        assert got.tolist() == want
    # unaligned base address (byte-load path)
    _native.xxh64_items(d[3:], n - 1, item_bytes, stride, out, 0)
    want = [xxhash.xxh64(buf[3 + i * stride:3 + i * stride + item_bytes].tobytes()).intdigest() for i in range(n - 1)]
    assert out[: n - 1].cpu().numpy().view(np.uint64).tolist() == want


def test_xxh64_many_items_and_one_long_item(cuda):
    """More item groups than SMs (the staged kernel's CTAs stride over groups; the
    last group is partial), and a single 1 MiB item (a long chunk sequence)."""
    rng = np.random.default_rng(99)
    n, L = 148 * 32 + 37, 1024
    buf = rng.integers(0, 256, n * L, dtype=np.uint8)
    out = torch.empty(n, dtype=torch.int64, device=cuda)
    _native.xxh64_items(torch.from_numpy(buf).to(cuda), n, L, L, out, 7)
    want = [xxhash.xxh64(buf[i * L:(i + 1) * L].tobytes(), seed=7).intdigest() for i in range(n)]
    assert out.cpu().numpy().view(np.uint64).tolist() == want
    big = rng.integers(0, 256, (1 << 20) + 3, dtype=np.uint8)
    one = torch.empty(1, dtype=torch.int64, device=cuda)
    _native.xxh64_items(torch.from_numpy(big).to(cuda), 1, big.size, big.size, one, 0)
    assert int(one.cpu().numpy().view(np.uint64)[0]) == xxhash.xxh64(big.tobytes()).intdigest()


def test_checksum_pages_of_kv_pages(cuda):
    pages = torch.randn(256, 16, 8, 128, device=cuda).to(torch.bfloat16)
    got = checksum_pages(pages).cpu().numpy().view(np.uint64)
    host = pages.cpu().view(torch.int16).numpy()
    for i in (0, 1, 100, 255):
        assert int(got[i]) == xxhash.xxh64(host[i].tobytes()).intdigest()
