"""Worker of tests/test_mg_gpu.py, run under torchrun: multi-GPU reduce, scan
and sort on NCCL ranks checked against the CPU oracle of the concatenated
input."""
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import oracle  # noqa: E402
from lc_parallel_primitive_b200 import _lib as L  # noqa: E402
from lc_parallel_primitive_b200 import datagen as G  # noqa: E402
from lc_parallel_primitive_b200 import multi_gpu as M  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ["LOCAL_RANK"]))
    dev = torch.device("cuda", int(os.environ["LOCAL_RANK"]))
    dist.init_process_group("nccl", device_id=dev)
    N = (1 << 22) + 12345
    bounds = [N * r // world for r in range(world + 1)]
    lo, hi = bounds[rank], bounds[rank + 1]
    # sort: u64 keys (config 5 shape, reduced n) + u32 values = global index
    keys = G.u64(N, seed=5, stream=1)
    vals = np.arange(N, dtype=np.uint32)
    r = M.mg_sort_pairs(torch.from_numpy(keys[lo:hi].view(np.int64)).to(dev).view(torch.uint64),
                        torch.from_numpy(vals[lo:hi].view(np.int32)).to(dev).view(torch.uint32))
    # duplicates-heavy keys (stability across ranks)
    kd = G.u32_masked(N, 0xF, seed=6)
    rd = M.mg_sort_pairs(torch.from_numpy(kd[lo:hi].view(np.int32)).to(dev).view(torch.uint32),
                         torch.from_numpy(vals[lo:hi].view(np.int32)).to(dev).view(torch.uint32))
    # scan + reduce
    xs = G.u32(N, seed=7)
    x = torch.from_numpy(xs[lo:hi].view(np.int32)).to(dev).view(torch.uint32)
    out = torch.empty_like(x)
    M.mg_scan(False, x, out)
    tot = M.mg_reduce(L.OP_SUM, x)
    mx = M.mg_reduce(L.OP_MAX, x)
    torch.cuda.synchronize()

    def gather_np(t, dtype):
        arr = t.cpu().numpy().view(dtype)
        objs = [None] * world
        dist.all_gather_object(objs, arr)
        return np.concatenate(objs)

    gk, gv = gather_np(r.keys.view(torch.int64), np.uint64), gather_np(r.values.view(torch.int32), np.uint32)
    dk, dv = gather_np(rd.keys.view(torch.int32), np.uint32), gather_np(rd.values.view(torch.int32), np.uint32)
    gs = gather_np(out.view(torch.int32), np.uint32)
    ok = True
    if rank == 0:
        wk, wv = oracle.radix_sort(keys, vals, threads=8)
        ok &= np.array_equal(gk, wk) and np.array_equal(gv, wv)
        wk, wv = oracle.radix_sort(kd, vals, threads=8)
        ok &= np.array_equal(dk, wk) and np.array_equal(dv, wv)
        ok &= np.array_equal(gs, oracle.scan(False, xs))
        ok &= int(tot.view(torch.int32).cpu()[0]) & 0xFFFFFFFF == int(oracle.reduce(0, xs))
        ok &= int(mx.view(torch.int32).cpu()[0]) & 0xFFFFFFFF == int(xs.max())
        print("MG_OK" if ok else "MG_FAIL", flush=True)
    dist.destroy_process_group()
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
