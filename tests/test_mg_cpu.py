"""Host logic of the multi-GPU primitives on 2 and 3 CPU ranks (gloo):
the orchestration of csrc/mg.cu restated step by step in
tests/mg_cpu_emulation.py (partition digit from the global key range,
bucket-to-rank plan from the library's lcpp_mg_sort_plan, rank-ordered
exchange, carries), checked against the oracle of the concatenated input."""
import ctypes as C
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _inputs(N):
    rng = np.random.default_rng(7)
    return {
        "dup": rng.integers(0, 50, size=N, dtype=np.uint32),               # many duplicates
        "u32": rng.integers(0, 1 << 32, size=N, dtype=np.uint64).astype(np.uint32),
        "u64": rng.integers(0, 1 << 63, size=N, dtype=np.uint64) * np.uint64(2) + np.uint64(1),
        "i32": rng.integers(-(1 << 31), 1 << 31, size=N, dtype=np.int64).astype(np.int32),
        "f32": rng.standard_normal(N).astype(np.float32),
        "masked": (rng.integers(0, 1 << 32, size=N, dtype=np.uint64) & np.uint64(0xF0F)).astype(np.uint32),
        "const": np.full(N, 12345, dtype=np.uint32),
        "scan": rng.integers(0, 1 << 32, size=N, dtype=np.uint64).astype(np.uint32),
    }


SORT_CASES = ["dup", "u32", "u64", "i32", "f32", "masked", "const"]


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from lc_parallel_primitive_b200 import _lib as L
        from tests import mg_cpu_emulation as E

        N = 10007
        data = _inputs(N)
        vals = np.arange(N, dtype=np.uint32)
        bounds = [N * r // world for r in range(world + 1)]
        lo, hi = bounds[rank], bounds[rank + 1]
        out = {}
        for name in SORT_CASES:
            k, v = E.mg_sort(data[name][lo:hi].copy(), vals[lo:hi].copy())
            out[name] = (k, v)
        xs = data["scan"][lo:hi].copy()
        out["scan"] = E.mg_scan(False, xs)
        out["max"] = E.mg_reduce(L.OP_MAX, xs)
        out["sum"] = E.mg_reduce(L.OP_SUM, xs)
        q.put((rank, out))
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
    got = [o for _, o in sorted([q.get(timeout=120) for _ in range(world)], key=lambda t: t[0])]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    N = 10007
    data = _inputs(N)
    vals = np.arange(N, dtype=np.uint32)
    from tests.mg_cpu_emulation import ordered_image

    for name in SORT_CASES:
        keys = data[name]
        order = np.argsort(ordered_image(keys), kind="stable")
        k = np.concatenate([g[name][0] for g in got])
        v = np.concatenate([g[name][1] for g in got])
        assert np.array_equal(k.view(keys.dtype), keys[order]), name
        assert np.array_equal(v, vals[order]), name  # global and stable
        sizes = [g[name][0].size for g in got]
        # extended-key splitters: even slices whatever the keys, duplicates included
        assert max(sizes) <= N / world * 1.06 + 8, (name, sizes)
    xs = data["scan"]
    scan = np.concatenate([g["scan"] for g in got])
    assert np.array_equal(scan, (np.cumsum(xs.astype(np.uint64)) - xs).astype(np.uint32))
    assert all(int(g["max"]) == int(xs.max()) for g in got)
    assert all(int(g["sum"]) == int(xs.astype(np.uint64).sum() & 0xFFFFFFFF) for g in got)


def test_mg_pick_splitters_weighted_quantiles():
    """The library's splitter choice (host export of the device rule): the
    sample where the running weight crosses r/G."""
    from tests.mg_cpu_emulation import pick_splitters

    keys = np.arange(100, dtype=np.uint64) * np.uint64(10)
    pos = np.arange(100, dtype=np.uint64)
    w = np.ones(100, dtype=np.uint64)
    k, p = pick_splitters(keys, pos, w, 4)
    assert k.tolist() == [250, 500, 750] and p.tolist() == [25, 50, 75]
    w2 = np.concatenate([np.full(50, 3, np.uint64), np.ones(50, np.uint64)])  # heavier first half
    k, _ = pick_splitters(keys, pos, w2, 2)
    assert k.tolist() == [330]  # running weight 100 of 200 is reached at sample 33
    k, p = pick_splitters(keys, pos, np.zeros(100, np.uint64), 3)  # no weight: sentinels
    assert k.tolist() == [2**64 - 1] * 2
    assert pick_splitters(keys, pos, w, 1)[0].size == 0
