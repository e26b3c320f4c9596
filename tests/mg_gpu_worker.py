"""Worker of tests/test_mg_gpu.py, run under torchrun: the multi-GPU C ABI
(lcpp_mg_reduce / lcpp_mg_scan / lcpp_mg_sort through multi_gpu.py) on NCCL
ranks, checked against the CPU oracle of the concatenated input."""
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

_SIGNED = {4: torch.int32, 8: torch.int64}


def dev_of(a: np.ndarray, dev):
    """Device tensor holding the array's bits (unsigned types through a signed view)."""
    return torch.from_numpy(np.ascontiguousarray(a).view(np.dtype(f"i{a.itemsize}"))).to(dev).view(
        {np.dtype(np.uint32): torch.uint32, np.dtype(np.uint64): torch.uint64, np.dtype(np.int32): torch.int32,
         np.dtype(np.int64): torch.int64, np.dtype(np.float32): torch.float32,
         np.dtype(np.float64): torch.float64}[a.dtype])


def host_of(t, dtype):
    return t.view(_SIGNED[t.element_size()]).cpu().numpy().view(dtype)


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev)
    comm = M.comm_for()
    N = (1 << 22) + 12345
    bounds = [N * r // world for r in range(world + 1)]
    lo, hi = bounds[rank], bounds[rank + 1]
    vals = np.arange(N, dtype=np.uint32)
    cases = {
        "u64": G.u64(N, seed=5, stream=1),                 # config 5 shape, reduced n
        "dup": G.u32_masked(N, 0xF, seed=6),               # 16 distinct keys: stability across ranks
        "f32": G.f32_normal(N, seed=8),                    # clustered float keys
        "const": np.full(N, 7, dtype=np.uint32),           # every key equal
    }
    results = {}
    for name, keys in cases.items():
        r = M.mg_sort_pairs(dev_of(keys[lo:hi], dev), dev_of(vals[lo:hi], dev), comm=comm)
        results[name] = (host_of(r.keys, keys.dtype), host_of(r.values, np.uint32))
    ko = M.mg_sort_pairs(dev_of(cases["u64"][lo:hi], dev), None, comm=comm)  # keys only
    results["keys_only"] = host_of(ko.keys, np.uint64)
    xs = G.u32(N, seed=7)
    x = dev_of(xs[lo:hi], dev)
    out = torch.empty_like(x)
    M.mg_scan(False, x, out, comm=comm)
    xf = G.f32_normal(N, seed=9)
    outf = torch.empty(hi - lo, dtype=torch.float32, device=dev)
    M.mg_scan(True, dev_of(xf[lo:hi], dev), outf, comm=comm)
    tot = M.mg_reduce(L.OP_SUM, x, comm=comm)
    mx = M.mg_reduce(L.OP_MAX, x, comm=comm)
    torch.cuda.synchronize()

    def gather(arr):
        objs = [None] * world
        dist.all_gather_object(objs, arr)
        return objs

    ok = True
    g = {name: gather(v) for name, v in results.items()}
    gs = np.concatenate(gather(host_of(out, np.uint32)))
    gf = np.concatenate(gather(outf.cpu().numpy()))
    if rank == 0:
        for name, keys in cases.items():
            wk, wv = oracle.radix_sort(keys, vals, threads=8)
            gk = np.concatenate([a for a, _ in g[name]])
            gv = np.concatenate([b for _, b in g[name]])
            good = np.array_equal(gk, wk) and np.array_equal(gv, wv)
            sizes = [a.size for a, _ in g[name]]
            good &= max(sizes) <= N / world * 1.06 + 8
            print(name, "ok" if good else "MISMATCH", sizes, flush=True)
            ok &= good
        ok &= np.array_equal(np.concatenate(g["keys_only"]), oracle.radix_sort(cases["u64"], threads=8))
        ok &= np.array_equal(gs, oracle.scan(False, xs))
        ref = np.cumsum(xf.astype(np.float64))
        ok &= bool(np.all(np.abs(gf - ref) <= 1e-5 * np.maximum(np.abs(ref), np.cumsum(np.abs(xf)) * 2.0 ** -10)))
        ok &= int(host_of(tot, np.uint32)[0]) == int(oracle.reduce(0, xs))
        ok &= int(host_of(mx, np.uint32)[0]) == int(xs.max())
        print(f"nranks={comm.nranks}", "MG_OK" if ok else "MG_FAIL", flush=True)
    M.destroy_comms()
    dist.destroy_process_group()
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
