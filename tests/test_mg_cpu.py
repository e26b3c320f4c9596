"""Host logic of the multi-GPU primitives on 2 and 3 CPU ranks (gloo), with
local passes done by the CPU stand-in: splitter choice, split counts,
all-to-all exchange, carries, rank-order stability."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from lc_parallel_primitive_b200 import _lib as L
        from lc_parallel_primitive_b200 import multi_gpu as M
        from tests.mg_cpu_ops import CpuOps

        ops = CpuOps()
        rng = np.random.default_rng(7)
        # global inputs, identical on every rank; shard r = contiguous slice r
        N = 10007
        keys = rng.integers(0, 50, size=N, dtype=np.uint32)  # many duplicates
        vals = np.arange(N, dtype=np.uint32)
        bounds = [N * r // world for r in range(world + 1)]
        lo, hi = bounds[rank], bounds[rank + 1]
        res = M.mg_sort_pairs(torch.from_numpy(keys[lo:hi].copy()), torch.from_numpy(vals[lo:hi].copy()), ops=ops)
        ukeys = rng.integers(0, 1 << 32, size=N, dtype=np.uint64).astype(np.uint32)  # balanced: bucket path
        ures = M.mg_sort_pairs(torch.from_numpy(ukeys[lo:hi].copy()), torch.from_numpy(vals[lo:hi].copy()), ops=ops)
        xs = rng.integers(0, 1 << 32, size=N, dtype=np.uint64).astype(np.uint32)
        out = torch.empty(hi - lo, dtype=torch.uint32)
        M.mg_scan(False, torch.from_numpy(xs[lo:hi].copy()), out, ops=ops)
        red = M.mg_reduce(L.OP_MAX, torch.from_numpy(xs[lo:hi].copy()), ops=ops)
        tot = M.mg_reduce(L.OP_SUM, torch.from_numpy(xs[lo:hi].copy()), ops=ops)
        q.put((rank, res.keys.numpy(), res.values.numpy(), res.counts_per_rank, out.numpy(), int(red[0]),
               int(tot.view(torch.int32)[0]) & 0xFFFFFFFF, ures.keys.numpy(), ures.values.numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_mg_host_logic_on_cpu_ranks(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = sorted([q.get(timeout=120) for _ in range(world)], key=lambda t: t[0])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    rng = np.random.default_rng(7)
    N = 10007
    keys = rng.integers(0, 50, size=N, dtype=np.uint32)
    vals = np.arange(N, dtype=np.uint32)
    ukeys = rng.integers(0, 1 << 32, size=N, dtype=np.uint64).astype(np.uint32)
    xs = rng.integers(0, 1 << 32, size=N, dtype=np.uint64).astype(np.uint32)
    uo = np.argsort(ukeys, kind="stable")
    assert np.array_equal(np.concatenate([g[7] for g in got]), ukeys[uo])
    assert np.array_equal(np.concatenate([g[8] for g in got]), vals[uo])
    order = np.argsort(keys, kind="stable")
    k = np.concatenate([g[1] for g in got])
    v = np.concatenate([g[2] for g in got])
    assert np.array_equal(k, keys[order]) and np.array_equal(v, vals[order])  # global, stable
    assert got[0][3] == [g[1].size for g in got]
    scan = np.concatenate([g[4] for g in got])
    want = (np.cumsum(xs.astype(np.uint64)) - xs).astype(np.uint32)
    assert np.array_equal(scan, want)
    assert all(g[5] == int(xs.max()) for g in got)
    assert all(g[6] == int(xs.astype(np.uint64).sum() & 0xFFFFFFFF) for g in got)
