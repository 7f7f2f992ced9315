"""Multi-rank host logic on CPU (gloo, world size 2): the pressure all-reduce
that keeps the replicated page-table policy identical on every rank."""
from __future__ import annotations

import os
import socket

import numpy as np
import torch.multiprocessing as mp

import oracle


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank: int, world: int, port: int, out) -> None:
    import sys
    from pathlib import Path
    repo = Path(__file__).resolve().parent.parent
    sys.path[:0] = [str(repo), str(repo / "ash-kv_b200")]
    import torch.distributed as dist
    from ashkv.runtime.distributed import allreduce_pressure
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    local = [0.5, 0.97][rank]
    p = allreduce_pressure(local)
    # every rank now evaluates the same thresholds on the same (replicated) features
    rng = np.random.default_rng(7)
    R = rng.random(4096, dtype=np.float32)
    cur = rng.integers(0, 4, 4096).astype(np.int8)
    nc, nh = oracle.controller_tables([(0, 1), (1, 0), (1, 2), (2, 1)])
    t = oracle.desired_tiers(R, cur, p, 0.72, 0.33, 0.04, 0.95, nc, nh)
    out.put((rank, p, t.tobytes()))
    dist.barrier()
    dist.destroy_process_group()


def test_pressure_allreduce_gloo_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    res.sort()
    assert res[0][1] == res[1][1] == np.float32(0.97)
    assert res[0][2] == res[1][2]  # identical tier decisions on both ranks


def test_allreduce_without_process_group_is_identity():
    import sys
    from pathlib import Path
    sys.path.insert(0, str(Path(__file__).resolve().parent.parent / "ash-kv_b200"))
    from ashkv.runtime.distributed import allreduce_pressure
    assert allreduce_pressure(0.42) == 0.42
