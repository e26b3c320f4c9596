"""Multi-GPU primitives on one node: one process per GPU, torch.distributed
(NCCL over NVLink/NVSwitch) for the exchange steps, this library's sm_100a
kernels (C ABI) for every local pass.  The reference has no multi-GPU support;
these follow the partitioning of its single-GPU semantics:

* mg_reduce          contiguous shards -> local DeviceReduce -> all_reduce of
                     one element per rank.
* mg_scan            contiguous shards -> local reduce -> all_gather of the G
                     shard totals -> carry = sum of the totals of lower ranks
                     -> local single-pass scan seeded with the carry
                     (12 bytes of HBM traffic per element).  Bit-exact for
                     integers (sums wrap mod 2^32 like the single-GPU scan).
* mg_sort_pairs      global stable sort of the concatenation of the shards in
                     rank order: one stable onesweep pass on the top 8 key
                     bits partitions each shard into 256 buckets -> the
                     all-reduced bucket counts assign contiguous bucket
                     ranges to ranks -> all_to_all of keys and values ->
                     full local onesweep sort of the received runs (stable,
                     and runs arrive in source-rank order, so equal keys keep
                     their global input order).  When the buckets cannot be
                     split evenly (skewed keys) each shard is fully sorted and
                     cut at sampled splitters instead (all keys equal to a
                     splitter go to the same rank).  Rank r ends up with the
                     r-th slice of the global order; slices are contiguous
                     and ordered but not equal in size.

Local work goes through an ``ops`` object: ``GpuOps`` (the default) calls the
CUDA kernels and fails loudly without them.  Tests of the host logic on CPU
ranks (gloo) pass a CPU implementation explicitly; the library never falls
back to one.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import _lib as L
from .primitives import lcpp_dtype

# ---------------------------------------------------------------------------
# Local operations on one GPU (C ABI)
# ---------------------------------------------------------------------------


class GpuOps:
    """Local passes on the current CUDA device through liblcpp_b200.so."""

    def __init__(self, stream=None):
        self.lib = L.lib()
        self.stream = stream

    def _s(self):
        return (self.stream or torch.cuda.current_stream()).cuda_stream

    @staticmethod
    def _tmp(nbytes, device):
        return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)

    def reduce(self, op: int, x: torch.Tensor) -> torch.Tensor:
        dt = lcpp_dtype(x)
        out = torch.empty(1, dtype=x.dtype, device=x.device)
        tb = self.lib.lcpp_reduce_temp_bytes(dt, x.numel())
        t = self._tmp(tb, x.device)
        L.check(self.lib.lcpp_reduce(op, dt, x.data_ptr(), out.data_ptr(), x.numel(), t.data_ptr(), tb, self._s()),
                "mg reduce")
        return out

    def scan(self, inclusive: bool, x: torch.Tensor, out: torch.Tensor, carry: torch.Tensor | None) -> None:
        dt = lcpp_dtype(x)
        tb = self.lib.lcpp_scan_temp_bytes(dt, x.numel())
        t = self._tmp(tb, x.device)
        L.check(self.lib.lcpp_scan_carry(int(inclusive), dt, x.data_ptr(), out.data_ptr(), x.numel(),
                                         None if carry is None else carry.data_ptr(), t.data_ptr(), tb, self._s()),
                "mg scan")

    def bucket_starts(self, keys: torch.Tensor, bit_start: int) -> torch.Tensor:
        """257 run boundaries of keys ordered by the 8-bit digit at bit_start."""
        out = torch.empty(257, dtype=torch.int64, device=keys.device)
        L.check(self.lib.lcpp_radix_bucket_starts(lcpp_dtype(keys), keys.data_ptr(), keys.numel(), bit_start,
                                                  out.data_ptr(), self._s()), "mg bucket starts")
        return out

    def sort_pairs(self, keys: torch.Tensor, vals: torch.Tensor, temp: torch.Tensor | None = None,
                   begin_bit: int = 0, end_bit: int = 0):
        kd, vd = lcpp_dtype(keys), lcpp_dtype(vals)
        n = keys.numel()
        ko, vo = torch.empty_like(keys), torch.empty_like(vals)
        if n == 0:
            return ko, vo
        tb = self.lib.lcpp_radix_sort_temp_bytes(kd, vd, n)
        t = temp if temp is not None and temp.numel() >= tb else self._tmp(tb, keys.device)
        L.check(self.lib.lcpp_radix_sort(kd, vd, 0, keys.data_ptr(), ko.data_ptr(), vals.data_ptr(), vo.data_ptr(),
                                         n, begin_bit, end_bit, t.data_ptr(), tb, self._s()), "mg sort")
        return ko, vo


# ---------------------------------------------------------------------------
# Order-preserving signed 64-bit image of keys (for splitters/searchsorted)
# ---------------------------------------------------------------------------
_SIGN64 = -(1 << 63)


def ordered_i64(keys: torch.Tensor) -> torch.Tensor:
    """int64 tensor whose signed order equals the keys' sort order (unsigned
    keys: flip the top bit of the 64-bit image; signed: widen)."""
    if keys.dtype in (torch.int32, torch.int64):
        return keys.to(torch.int64)
    if keys.dtype == torch.uint32:
        return keys.view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    if keys.dtype == torch.uint64:
        return keys.view(torch.int64) ^ _SIGN64
    raise TypeError(f"mg_sort_pairs: unsupported key type {keys.dtype}")


def _all_gather_1d(x: torch.Tensor, group=None) -> torch.Tensor:
    """Concatenation of every rank's equally sized 1-D tensor, in rank order."""
    world = dist.get_world_size(group)
    parts = [torch.empty_like(x) for _ in range(world)]
    dist.all_gather(parts, x.contiguous(), group=group)
    return torch.cat(parts)


def _op_to_reduce_op(op: int):
    return {L.OP_SUM: dist.ReduceOp.SUM, L.OP_MIN: dist.ReduceOp.MIN, L.OP_MAX: dist.ReduceOp.MAX}[op]


# ---------------------------------------------------------------------------
def mg_reduce(op: int, x_local: torch.Tensor, ops=None, group=None) -> torch.Tensor:
    """Reduction of the concatenation of all ranks' shards (result on every rank)."""
    ops = ops or GpuOps()
    part = ops.reduce(op, x_local)
    if part.dtype == torch.uint32:  # collectives on 32-bit unsigned: sum wraps identically on int32 bits;
        if op == L.OP_SUM:         # min/max compare on the zero-extended int64 image
            p = part.view(torch.int32).clone()
            dist.all_reduce(p, op=dist.ReduceOp.SUM, group=group)
            return p.view(torch.uint32)
        p = part.view(torch.int32).to(torch.int64) & 0xFFFFFFFF
        dist.all_reduce(p, op=_op_to_reduce_op(op), group=group)
        return p.to(torch.int32).view(torch.uint32)
    p = part.clone()
    dist.all_reduce(p, op=_op_to_reduce_op(op), group=group)
    return p


def shard_carry(totals: torch.Tensor, rank: int) -> torch.Tensor:
    """Exclusive sum of the shard totals of ranks below `rank` (wrapping for
    32-bit integers), as a 1-element tensor of the totals' dtype."""
    if totals.dtype in (torch.int32, torch.uint32):
        t = totals.view(torch.int32).to(torch.int64)[:rank].sum() & 0xFFFFFFFF
        c = t.to(torch.int64).reshape(1)
        c = torch.where(c >= (1 << 31), c - (1 << 32), c).to(torch.int32)
        return c.view(totals.dtype)
    return totals[:rank].sum().reshape(1).to(totals.dtype)


def mg_scan(inclusive: bool, x_local: torch.Tensor, out_local: torch.Tensor, ops=None, group=None) -> None:
    """Prefix sum of the concatenation of all ranks' shards, in rank order."""
    ops = ops or GpuOps()
    rank = dist.get_rank(group)
    total = ops.reduce(L.OP_SUM, x_local)
    if total.dtype == torch.uint32:
        gathered = _all_gather_1d(total.view(torch.int32), group).view(torch.uint32)
    else:
        gathered = _all_gather_1d(total, group)
    carry = shard_carry(gathered, rank)
    ops.scan(inclusive, x_local, out_local, carry if rank > 0 else None)


@dataclass
class SortResult:
    keys: torch.Tensor
    values: torch.Tensor
    counts_per_rank: list  # number of elements that ended on each rank (all_gathered)


def choose_splitters(samples_sorted_i64: torch.Tensor, world: int) -> torch.Tensor:
    """G-1 splitters from the globally sorted sample: every (len/G)-th sample."""
    m = samples_sorted_i64.numel()
    if world == 1 or m == 0:
        return samples_sorted_i64.new_empty(0)
    idx = torch.arange(1, world, device=samples_sorted_i64.device) * m // world
    return samples_sorted_i64[idx]


def split_counts(sorted_keys_i64: torch.Tensor, splitters: torch.Tensor) -> torch.Tensor:
    """Elements of a sorted shard that go to each rank: rank r receives keys
    in [splitter[r-1], splitter[r]) (first rank from -inf, last to +inf)."""
    n = sorted_keys_i64.numel()
    cuts = torch.searchsorted(sorted_keys_i64, splitters, right=False) if splitters.numel() else \
        splitters.new_empty(0)
    bounds = torch.cat([cuts.new_zeros(1), cuts, cuts.new_full((1,), n)])
    return (bounds[1:] - bounds[:-1]).to(torch.int64)


def rank_bucket_ranges(global_counts: list, world: int):
    """Split the 256 top-byte buckets into `world` contiguous ranges of about
    equal element count.  Returns (bucket boundaries[world+1], max load / mean load)."""
    total = sum(global_counts)
    cum, acc = [], 0
    for c in global_counts:
        acc += c
        cum.append(acc)
    bounds = [0]
    for r in range(1, world):
        target = total * r / world
        # first bucket whose end overshoots the target starts rank r, unless
        # stopping before it is closer to the target
        b = next((i for i, e in enumerate(cum) if e > target), 256)
        before = cum[b - 1] if b > 0 else 0
        if b < 256 and cum[b] - target < target - before:
            b += 1
        bounds.append(max(b, bounds[-1]))
    bounds.append(256)
    loads = [(cum[bounds[r + 1] - 1] if bounds[r + 1] > 0 else 0) - (cum[bounds[r] - 1] if bounds[r] > 0 else 0)
             for r in range(world)]
    mean = total / world if world else 0
    return bounds, (max(loads) / mean if mean else 1.0)


def _exchange(k1, v1, send_counts, keys_dtype, vals_dtype, group):
    """Send send_counts[r] consecutive (key, value) pairs to rank r; receive
    the runs of every rank, concatenated in source-rank order.  Keys and
    values travel as raw bits in one batch of NCCL point-to-point calls."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    recv_counts = torch.empty_like(send_counts)
    dist.all_to_all_single(recv_counts, send_counts, group=group)
    sc = send_counts.cpu().tolist()
    rc = recv_counts.cpu().tolist()
    kview = torch.int64 if k1.element_size() == 8 else torch.int32
    vview = torch.int64 if v1.element_size() == 8 else torch.int32
    rk = torch.empty(int(sum(rc)), dtype=kview, device=k1.device)
    rv = torch.empty(int(sum(rc)), dtype=vview, device=k1.device)
    ks, vs = k1.view(kview), v1.view(vview)
    so, ro = [0], [0]
    for c in sc:
        so.append(so[-1] + c)
    for c in rc:
        ro.append(ro[-1] + c)
    p2p = []
    for p in range(world):
        if p == rank:
            continue
        peer = dist.get_global_rank(group, p) if group is not None else p
        if sc[p]:
            p2p.append(dist.P2POp(dist.isend, ks[so[p]:so[p + 1]], peer, group))
            p2p.append(dist.P2POp(dist.isend, vs[so[p]:so[p + 1]], peer, group))
        if rc[p]:
            p2p.append(dist.P2POp(dist.irecv, rk[ro[p]:ro[p + 1]], peer, group))
            p2p.append(dist.P2POp(dist.irecv, rv[ro[p]:ro[p + 1]], peer, group))
    rk[ro[rank]:ro[rank + 1]].copy_(ks[so[rank]:so[rank + 1]])
    rv[ro[rank]:ro[rank + 1]].copy_(vs[so[rank]:so[rank + 1]])
    if p2p:
        for w in dist.batch_isend_irecv(p2p):
            w.wait()
    return rk.view(keys_dtype), rv.view(vals_dtype)


def mg_sort_pairs(keys_local: torch.Tensor, vals_local: torch.Tensor, ops=None, group=None,
                  samples_per_rank: int = 1024, max_imbalance: float = 1.25) -> SortResult:
    """Globally stable sort of (keys, values) sharded over the ranks in rank
    order.  Returns this rank's slice of the sorted sequence.

    Fast path: one stable onesweep pass on the top 8 key bits partitions the
    shard; an all-reduced 256-bin count assigns contiguous bucket ranges to
    ranks; if that split is balanced (max load <= max_imbalance x mean) the
    buckets are exchanged and each rank sorts what it received.  Otherwise
    (skewed keys) the shard is fully sorted and cut at sampled splitters.
    """
    ops = ops or GpuOps()
    world = dist.get_world_size(group)
    if world == 1:
        k1, v1 = ops.sort_pairs(keys_local, vals_local)
        return SortResult(k1, v1, [k1.numel()])
    dev = keys_local.device
    kbits = keys_local.element_size() * 8
    k1, v1 = ops.sort_pairs(keys_local, vals_local, begin_bit=kbits - 8, end_bit=kbits)  # partition pass
    n = k1.numel()
    starts = ops.bucket_starts(k1, kbits - 8)  # 257 run boundaries
    global_counts = torch.diff(starts)
    dist.all_reduce(global_counts, group=group)
    bounds, imbalance = rank_bucket_ranges(global_counts.cpu().tolist(), world)
    if imbalance <= max_imbalance:
        send_counts = torch.diff(starts[torch.tensor(bounds, device=dev)]).to(torch.int64)
    else:
        k1, v1 = ops.sort_pairs(k1, v1)  # full local sort (stable: partition kept input order)
        ki = ordered_i64(k1)
        s = min(samples_per_rank, max(n, 1))
        if n:
            samp = ki[(torch.arange(s, device=dev, dtype=torch.int64) * n) // s]
        else:
            samp = torch.full((s,), torch.iinfo(torch.int64).max, dtype=torch.int64, device=dev)
        all_samp, _ = torch.sort(_all_gather_1d(samp, group))  # G*s samples: tiny
        send_counts = split_counts(ki, choose_splitters(all_samp, world))
        del ki
    rk, rv = _exchange(k1, v1, send_counts, keys_local.dtype, vals_local.dtype, group)
    del k1, v1
    k2, v2 = ops.sort_pairs(rk, rv)  # final local sort of the received runs
    all_counts = _all_gather_1d(torch.tensor([rk.numel()], dtype=torch.int64, device=dev), group)
    return SortResult(k2, v2, all_counts.cpu().tolist())
