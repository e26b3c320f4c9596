"""Multi-GPU primitives on one node (one process per GPU): a binding of the
library's C ABI (lcpp_mg_reduce, lcpp_mg_scan, lcpp_mg_sort in
include/lcpp_b200.h), which runs every local pass as an sm_100a kernel and
every exchange as an NCCL call on an NCCL communicator the library builds.
torch.distributed only carries the communicator's unique id from rank 0 to
the other ranks; the data path never goes through it.

The reference has no multi-GPU support; these extend its single-GPU
DeviceReduce / DeviceScan / DeviceRadixSort (src/lcpp/device/
device_reduce.h:169-185, device_scan.h:180-204, device_radix_sort.h:129-153)
to shards held in rank order:

* mg_reduce      local reduce -> NCCL all-reduce of one element.
* mg_scan        local reduce -> all-gather of the G shard totals -> carry
                 (sum of lower ranks' totals, in rank order) -> local scan
                 seeded with the carry.  No host synchronisation.
* mg_sort_pairs  global stable sort: 4096 samples per rank of the extended
                 key (key, rank, index), all-gathered and sorted on the device
                 -> G-1 splitters -> destination byte per item -> one stable
                 onesweep pass over those bytes -> grouped NCCL send/recv ->
                 local onesweep sort of the key bits that differ.  One host
                 synchronisation (the exchange sizes).  Rank r gets the r-th
                 contiguous slice of the global order, about n_total/G items
                 whatever the key distribution.

Scratch comes from a caller temp tensor sized by the *_temp_bytes functions
(or is allocated once per call when none is passed).  There is no CPU path:
without the CUDA library or NCCL every call raises.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import _lib as L
from .primitives import lcpp_dtype

_COMMS: dict = {}


class MgComm:
    """An NCCL communicator over the ranks of a torch.distributed group, made
    by liblcpp_b200 (ncclGetUniqueId on the group's first rank, broadcast of
    the id, ncclCommInitRank on every rank).  The current CUDA device of each
    process is its rank's GPU."""

    def __init__(self, group=None):
        lib = L.lib()
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        nbytes = int(lib.lcpp_mg_unique_id_bytes())
        buf = C.create_string_buffer(nbytes)
        if self.rank == 0:
            L.check(lib.lcpp_mg_get_unique_id(buf), "ncclGetUniqueId")
        obj = [buf.raw if self.rank == 0 else None]
        src = dist.get_global_rank(group, 0) if group is not None else 0
        dist.broadcast_object_list(obj, src=src, group=group)
        buf = C.create_string_buffer(obj[0], nbytes)
        handle = C.c_void_p()
        L.check(lib.lcpp_mg_comm_init_rank(C.byref(handle), self.world, buf, self.rank), "ncclCommInitRank")
        self.handle = handle
        r, n = C.c_int(), C.c_int()
        L.check(lib.lcpp_mg_comm_shape(self.handle, C.byref(r), C.byref(n)), "ncclCommCount")
        self.nranks = n.value
        assert r.value == self.rank and n.value == self.world, "communicator does not match the group"

    def close(self) -> None:
        if self.handle:
            L.check(L.lib().lcpp_mg_comm_destroy(self.handle), "ncclCommDestroy")
            self.handle = None


def comm_for(group=None) -> MgComm:
    """The (cached) library communicator of a torch.distributed group."""
    key = id(group) if group is not None else None
    c = _COMMS.get(key)
    if c is None or c.handle is None:
        c = MgComm(group)
        _COMMS[key] = c
    return c


def destroy_comms() -> None:
    for c in _COMMS.values():
        c.close()
    _COMMS.clear()


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _temp(temp, nbytes, device):
    if temp is not None:
        if temp.numel() * temp.element_size() < nbytes:
            raise ValueError(f"temp holds {temp.numel() * temp.element_size()} bytes, {nbytes} needed")
        return temp
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)


# ---------------------------------------------------------------------------
def mg_reduce_temp_bytes(x_local: torch.Tensor) -> int:
    return int(L.lib().lcpp_mg_reduce_temp_bytes(lcpp_dtype(x_local), x_local.numel()))


def mg_reduce(op: int, x_local: torch.Tensor, comm: MgComm | None = None, temp=None,
              out: torch.Tensor | None = None) -> torch.Tensor:
    """op (L.OP_SUM / OP_MIN / OP_MAX) over the concatenation of all ranks'
    shards; the 1-element result is on every rank."""
    comm = comm or comm_for()
    lib = L.lib()
    dt = lcpp_dtype(x_local)
    out = torch.empty(1, dtype=x_local.dtype, device=x_local.device) if out is None else out
    tb = mg_reduce_temp_bytes(x_local)
    t = _temp(temp, tb, x_local.device)
    L.check(lib.lcpp_mg_reduce(op, dt, x_local.data_ptr(), out.data_ptr(), x_local.numel(), t.data_ptr(),
                               t.numel() * t.element_size(), comm.handle, _stream()), "mg_reduce")
    return out


def mg_scan_temp_bytes(x_local: torch.Tensor, world: int) -> int:
    return int(L.lib().lcpp_mg_scan_temp_bytes(lcpp_dtype(x_local), x_local.numel(), world))


def mg_scan(inclusive: bool, x_local: torch.Tensor, out_local: torch.Tensor, comm: MgComm | None = None,
            temp=None) -> None:
    """Prefix sum of the concatenation of all ranks' shards, in rank order;
    each rank writes its own shard's part into out_local."""
    comm = comm or comm_for()
    lib = L.lib()
    tb = mg_scan_temp_bytes(x_local, comm.world)
    if tb == 0:
        raise L.LcppError(L.ERR_INVALID_ARG, f"mg_scan: unsupported dtype {x_local.dtype}")
    t = _temp(temp, tb, x_local.device)
    L.check(lib.lcpp_mg_scan(int(inclusive), lcpp_dtype(x_local), x_local.data_ptr(), out_local.data_ptr(),
                             x_local.numel(), t.data_ptr(), t.numel() * t.element_size(), comm.handle, _stream()),
            "mg_scan")


@dataclass
class SortResult:
    keys: torch.Tensor     # this rank's slice of the sorted global sequence
    values: torch.Tensor | None
    n: int                 # its length


def default_capacity(n_local: int) -> int:
    """Output room per rank: the sampled splitters put about n_total/G items
    on every rank (within a few percent at 4096 samples per rank), so 1/8
    above the shard size covers even shards; a slice that still does not fit
    raises with ERR_CAPACITY."""
    return min(n_local + max(n_local // 8, 4096), (1 << 32) - 1)


def mg_sort_temp_bytes(keys: torch.Tensor, values: torch.Tensor | None, capacity: int, world: int) -> int:
    vd = L.NONE if values is None else lcpp_dtype(values)
    return int(L.lib().lcpp_mg_sort_temp_bytes(lcpp_dtype(keys), vd, keys.numel(), capacity, world))


def mg_sort_pairs(keys_local: torch.Tensor, vals_local: torch.Tensor | None, comm: MgComm | None = None,
                  capacity: int | None = None, temp=None, keys_out=None, vals_out=None) -> SortResult:
    """Global stable ascending sort of (key, value) pairs sharded over the
    ranks in rank order (vals_local None: keys only).  Returns this rank's
    contiguous slice of the sorted sequence (views of keys_out/vals_out)."""
    comm = comm or comm_for()
    lib = L.lib()
    n = keys_local.numel()
    cap = default_capacity(n) if capacity is None else int(capacity)
    dev = keys_local.device
    ko = torch.empty(max(cap, 1), dtype=keys_local.dtype, device=dev) if keys_out is None else keys_out
    vo = None
    if vals_local is not None:
        vo = torch.empty(max(cap, 1), dtype=vals_local.dtype, device=dev) if vals_out is None else vals_out
    if ko.numel() < cap or (vo is not None and vo.numel() < cap):
        raise ValueError("output buffers are smaller than capacity")
    tb = mg_sort_temp_bytes(keys_local, vals_local, cap, comm.world)
    if tb == 0:
        raise L.LcppError(L.ERR_INVALID_ARG, f"mg_sort_pairs: unsupported key type {keys_local.dtype}")
    t = _temp(temp, tb, dev)
    n_out = C.c_uint64(0)
    vd = L.NONE if vals_local is None else lcpp_dtype(vals_local)
    L.check(lib.lcpp_mg_sort(lcpp_dtype(keys_local), vd, keys_local.data_ptr(),
                             None if vals_local is None else vals_local.data_ptr(), n, ko.data_ptr(),
                             None if vo is None else vo.data_ptr(), cap, C.byref(n_out), t.data_ptr(),
                             t.numel() * t.element_size(), comm.handle, _stream()), "mg_sort")
    m = int(n_out.value)
    return SortResult(ko[:m], None if vo is None else vo[:m], m)
