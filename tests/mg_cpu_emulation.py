"""Step-by-step CPU restatement of the multi-GPU orchestration in
lc_parallel_primitive_b200/csrc/mg.cu, run on gloo ranks by
tests/test_mg_cpu.py.  The local passes are the oracle's; the bucket-to-rank
assignment is the library's own (lcpp_mg_sort_plan, the host export of the
function the device plan kernel runs); the collectives are the ones mg.cu
issues through NCCL (all-reduce of {min, ~max}, all-gather of the bucket
starts / shard totals, point-to-point exchange in rank order).  Test
infrastructure only."""
import ctypes as C

import numpy as np
import torch
import torch.distributed as dist

import oracle
from lc_parallel_primitive_b200 import _lib as L

_UNS = {np.dtype(np.uint32): np.uint32, np.dtype(np.int32): np.uint32, np.dtype(np.float32): np.uint32,
        np.dtype(np.uint64): np.uint64, np.dtype(np.int64): np.uint64, np.dtype(np.float64): np.uint64}


def ordered_image(k: np.ndarray) -> np.ndarray:
    """Order-preserving unsigned image of the keys (the sort's key twiddle)."""
    u = _UNS[k.dtype]
    bits = k.view(u).astype(np.uint64)
    w = k.dtype.itemsize * 8
    high = np.uint64(1 << (w - 1))
    allb = np.uint64((1 << w) - 1)
    if k.dtype.kind == "u":
        return bits
    if k.dtype.kind == "i":
        return bits ^ high
    o = np.where(bits & high, (~bits) & allb, bits ^ high)
    return np.where(o == (high - np.uint64(1)), high, o)  # -0.0 as +0.0


_SIGNED = {1: np.int8, 2: np.int16, 4: np.int32, 8: np.int64}


def _wire(arr: np.ndarray) -> torch.Tensor:
    """Tensor over the array's bits as a signed type (gloo carries no unsigned types)."""
    return torch.from_numpy(np.ascontiguousarray(arr).view(_SIGNED[arr.dtype.itemsize]))


def _allgather(arr: np.ndarray) -> np.ndarray:
    t = _wire(arr)
    parts = [torch.empty_like(t) for _ in range(dist.get_world_size())]
    dist.all_gather(parts, t)
    return np.stack([p.numpy().view(arr.dtype) for p in parts])


def mg_reduce(op, x):
    part = np.array([oracle.reduce(op, x)], dtype=x.dtype)
    allp = _allgather(part)[:, 0]
    return oracle.reduce(op, allp)


def mg_scan(inclusive, x):
    me = dist.get_rank()
    total = np.array([oracle.reduce(L.OP_SUM, x)], dtype=x.dtype)
    totals = _allgather(total)[:, 0]
    carry = totals[:me].astype(np.uint64).sum() if x.dtype.kind in "iu" else totals[:me].sum()
    y = oracle.scan(inclusive, x)
    if x.dtype.kind in "iu":
        return (y.astype(np.uint64) + np.uint64(carry)).astype(x.dtype)
    return (y + x.dtype.type(carry)).astype(x.dtype)


MG_SAMPLES = 4096  # per rank, as csrc/mg.cu


def _u64(arr):
    return np.ascontiguousarray(arr, dtype=np.uint64).ctypes.data_as(C.POINTER(C.c_uint64))


def pick_splitters(skey, spos, sw, G):
    """The library's splitter choice (lcpp_mg_pick_splitters) on sorted samples."""
    sk, sp, w = (np.ascontiguousarray(x, dtype=np.uint64) for x in (skey, spos, sw))
    ok_, op_ = np.zeros(max(G - 1, 1), np.uint64), np.zeros(max(G - 1, 1), np.uint64)
    L.check(L.lib().lcpp_mg_pick_splitters(_u64(sk), _u64(sp), _u64(w), sk.size, G,
                                           ok_.ctypes.data_as(C.POINTER(C.c_uint64)),
                                           op_.ctypes.data_as(C.POINTER(C.c_uint64))))
    return ok_[:G - 1], op_[:G - 1]


def mg_sort(keys, vals):
    """Rank's slice of the global stable sort, computed like lcpp_mg_sort."""
    G, me = dist.get_world_size(), dist.get_rank()
    n = keys.size
    if G == 1:
        return oracle.radix_sort(keys, vals)
    o = ordered_image(keys)
    # global min / max of the image -> bits that still differ (the library reduces
    # it in its bucket kernel and all-reduces it with the bucket starts; the
    # value is the same)
    lo = int(o.min()) if n else (1 << 64) - 1
    nhi = int(~o.max() & np.uint64((1 << 64) - 1)) if n else (1 << 64) - 1
    sign = np.uint64(1 << 63)
    mm = torch.from_numpy((np.array([lo, nhi], dtype=np.uint64) ^ sign).view(np.int64))  # unsigned order as signed
    dist.all_reduce(mm, op=dist.ReduceOp.MIN)
    g = mm.numpy().view(np.uint64) ^ sign
    x = int(g[0]) ^ (~int(g[1]) & ((1 << 64) - 1))
    hb = x.bit_length() - 1
    #    samples of extended keys, gathered rank-major, stably sorted by key
    if n:
        p = (np.arange(MG_SAMPLES, dtype=np.uint64) * np.uint64(n)) // np.uint64(MG_SAMPLES)
        sk, sp = o[p.astype(np.int64)], (np.uint64(me) << np.uint64(32)) | p
        sw = np.full(MG_SAMPLES, n, dtype=np.uint64)
    else:
        sk = sp = np.full(MG_SAMPLES, (1 << 64) - 1, dtype=np.uint64)
        sw = np.zeros(MG_SAMPLES, dtype=np.uint64)
    ak, ap, aw = (_allgather(v).reshape(-1) for v in (sk, sp, sw))
    order = np.argsort(ak, kind="stable")
    spk, spp = pick_splitters(ak[order], ap[order], aw[order], G)
    # 2. destination of every item = number of splitters <= its extended key
    pos = (np.uint64(me) << np.uint64(32)) | np.arange(n, dtype=np.uint64)
    dest = np.zeros(n, dtype=np.int64)
    for k_, p_ in zip(spk, spp):
        dest += ((k_ < o) | ((k_ == o) & (p_ <= pos))).astype(np.int64)
    perm = np.argsort(dest, kind="stable")
    pk, pv = keys[perm], vals[perm]
    starts = np.searchsorted(dest[perm], np.arange(G + 1), side="left").astype(np.int64)
    # 3. all-gathered starts -> exchange sizes
    rows = _allgather(starts)
    so = starts.tolist()
    rc = [int(rows[p_, me + 1] - rows[p_, me]) for p_ in range(G)]
    # 4. exchange: runs in source-rank order
    ks, vs = [None] * G, [None] * G
    reqs = []
    for p in range(G):
        if p == me:
            ks[p], vs[p] = pk[so[p]:so[p + 1]], pv[so[p]:so[p + 1]]
            continue
        sk, sv = _wire(pk[so[p]:so[p + 1]]), _wire(pv[so[p]:so[p + 1]])
        rk, rv = _wire(np.empty(rc[p], dtype=keys.dtype)), _wire(np.empty(rc[p], dtype=vals.dtype))
        ks[p], vs[p] = rk, rv
        for t in (sk, sv):
            if t.numel():
                reqs.append(dist.isend(t, p))
        for t in (rk, rv):
            if t.numel():
                reqs.append(dist.irecv(t, p))
    for r in reqs:
        r.wait()
    rk = np.concatenate([np.asarray(k).view(keys.dtype) for k in ks])
    rv = np.concatenate([np.asarray(v).view(vals.dtype) for v in vs])
    # 5. local sort of the differing bits
    if hb < 0 or rk.size == 0:
        return rk, rv
    return oracle.radix_sort(rk, rv, begin_bit=0, end_bit=hb + 1)
