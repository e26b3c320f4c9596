"""Python host mirror of LCPP's public Device* classes, over the C ABI.

Same class names, method names, argument order and meaning as the reference's
C++ templates (namespace luisa::parallel_primitive):

  DeviceReduce        src/lcpp/device/device_reduce.h:41-325 (incl. ArgMin/ArgMax, ReduceByKey)
  DeviceScan          src/lcpp/device/device_scan.h:33-345 (incl. ScanByKey)
  DeviceRadixSort     src/lcpp/device/device_radix_sort.h:37-184
  DeviceSegmentReduce src/lcpp/device/device_segment_reduce.h:26-194

Buffers are CUDA torch tensors (torch provides device memory and streams
only).  As in the reference, calls are recorded into a CommandList and run
when the list is committed to a Stream:

    stream << cmdlist.commit() << synchronize()

Error behaviour: the reference's lcpp_check asserts in debug builds and is a
no-op in release (src/lcpp/runtime/core.h:57-66); this mirror always raises
LcppError on a non-zero status.  No CPU fallback exists: without the built
liblcpp_b200.so every call raises.
"""
from __future__ import annotations

from typing import Callable, List, Optional

import torch

from . import _lib as L

_DTYPES = {
    torch.int32: L.I32,
    torch.uint32: L.U32,
    torch.float32: L.F32,
    torch.int64: L.I64,
    torch.uint64: L.U64,
    torch.float64: L.F64,
}


def lcpp_dtype(t) -> int:
    dt = t.dtype if isinstance(t, torch.Tensor) else t
    try:
        return _DTYPES[dt]
    except KeyError:
        raise TypeError(f"unsupported element type {dt}") from None


_NP = {L.I32: "int32", L.U32: "uint32", L.F32: "float32", L.I64: "int64", L.U64: "uint64", L.F64: "float64"}


def _host_scalar(value, dt):
    """One element of lcpp dtype `dt` in host memory (kept alive by the caller)."""
    import numpy as np

    return np.array([value], dtype=_NP[dt])


def _op_code(op) -> int:
    return {"sum": L.OP_SUM, "min": L.OP_MIN, "max": L.OP_MAX}[op] if isinstance(op, str) else int(op)


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("buffers must be CUDA tensors")
    if not t.is_contiguous():
        raise ValueError("buffers must be contiguous")
    return t.data_ptr()


def _nbytes(t: Optional[torch.Tensor]) -> int:
    return 0 if t is None else t.numel() * t.element_size()


def _stream_handle(stream) -> int:
    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, Stream):
        return stream.torch_stream.cuda_stream
    return stream.cuda_stream


# ---------------------------------------------------------------------------
# Minimal runtime shim: Stream / CommandList / synchronize
# ---------------------------------------------------------------------------
class _Commit:
    def __init__(self, cmds):
        self.cmds = cmds


class _Sync:
    pass


def synchronize() -> _Sync:
    return _Sync()


class CommandList:
    """Deferred commands; each is a callable taking the CUDA stream handle."""

    def __init__(self):
        self._cmds: List[Callable[[int], None]] = []

    def append(self, fn: Callable[[int], None]) -> None:
        self._cmds.append(fn)

    def __lshift__(self, fn):
        self.append(fn)
        return self

    def __len__(self):
        return len(self._cmds)

    def commit(self) -> _Commit:
        cmds, self._cmds = self._cmds, []
        return _Commit(cmds)


class Stream:
    def __init__(self, torch_stream: Optional[torch.cuda.Stream] = None):
        self.torch_stream = torch_stream or torch.cuda.current_stream()

    def __lshift__(self, item):
        if isinstance(item, _Commit):
            h = self.torch_stream.cuda_stream
            for c in item.cmds:
                c(h)
        elif isinstance(item, _Sync):
            self.torch_stream.synchronize()
        elif callable(item):
            item(self.torch_stream.cuda_stream)
        else:
            raise TypeError(f"cannot submit {type(item)} to a Stream")
        return self

    def synchronize(self):
        self.torch_stream.synchronize()


class _Module:
    """Common part of the Device* classes (create + template parameters)."""

    def __init__(self, BLOCK_SIZE: int = 256, WARP_NUMS: int = 32, ITEMS_PER_THREAD: int = 4):
        # Kept for API compatibility; tuning is internal to the sm_100a kernels.
        self.BLOCK_SIZE, self.WARP_NUMS, self.ITEMS_PER_THREAD = BLOCK_SIZE, WARP_NUMS, ITEMS_PER_THREAD
        self._device = None
        self._debug_stream = None

    def create(self, device=None, debug_stream: Optional[Stream] = None) -> None:
        L.lib()  # fail loudly now if the native library is missing
        self._device = device
        self._debug_stream = debug_stream

    def _record(self, cmdlist: CommandList, fn: Callable[[int], int], what: str) -> None:
        def run(stream_handle: int):
            L.check(fn(stream_handle), what)

        cmdlist.append(run)
        if self._debug_stream is not None:  # debug: commit + synchronize at once
            self._debug_stream << cmdlist.commit() << synchronize()


# ---------------------------------------------------------------------------
class DeviceReduce(_Module):
    @staticmethod
    def GetTempStorageBytes(num_item: int, dtype=torch.int32) -> int:
        return int(L.lib().lcpp_reduce_temp_bytes(lcpp_dtype(dtype), num_item))

    def Reduce(self, cmdlist, temp_storage, d_in, d_out, num_item, op: int):
        dt = lcpp_dtype(d_in)
        if lcpp_dtype(d_out) != dt:
            raise TypeError("d_in and d_out must have the same element type")
        pin, pout, ptmp, nt = _ptr(d_in), _ptr(d_out), _ptr(temp_storage), _nbytes(temp_storage)
        self._record(cmdlist, lambda s: L.lib().lcpp_reduce(op, dt, pin, pout, num_item, ptmp, nt, s),
                     "DeviceReduce")

    def Sum(self, cmdlist, temp_storage, d_in, d_out, num_item):
        self.Reduce(cmdlist, temp_storage, d_in, d_out, num_item, L.OP_SUM)

    def Min(self, cmdlist, temp_storage, d_in, d_out, num_item):
        self.Reduce(cmdlist, temp_storage, d_in, d_out, num_item, L.OP_MIN)

    def Max(self, cmdlist, temp_storage, d_in, d_out, num_item):
        self.Reduce(cmdlist, temp_storage, d_in, d_out, num_item, L.OP_MAX)

    def TransformReduce(self, cmdlist, temp_storage, d_in, d_out, num_item, reduce_op, transform_op, init):
        """reduce_op: "sum" | "min" | "max"; transform_op: "identity" | "square" | "abs" | "negate"
        (the reference's DSL lambdas, device_reduce.h:331-348); out = reduce_op(init, reduce(transform(x)))."""
        dt = lcpp_dtype(d_in)
        if lcpp_dtype(d_out) != dt:
            raise TypeError("d_in and d_out must have the same element type")
        op = _op_code(reduce_op)
        xf = {"identity": L.XF_IDENTITY, "square": L.XF_SQUARE, "abs": L.XF_ABS,
              "negate": L.XF_NEGATE}[transform_op] if isinstance(transform_op, str) else int(transform_op)
        iv = _host_scalar(init, dt)
        pin, pout, ptmp, nt = _ptr(d_in), _ptr(d_out), _ptr(temp_storage), _nbytes(temp_storage)
        self._record(cmdlist,
                     lambda s: L.lib().lcpp_transform_reduce(op, xf, dt, pin, pout, num_item, iv.ctypes.data, ptmp,
                                                             nt, s),
                     "DeviceReduce.TransformReduce")

    @staticmethod
    def GetArgTempStorageBytes(num_item: int, dtype=torch.int32) -> int:
        return int(L.lib().lcpp_arg_reduce_temp_bytes(lcpp_dtype(dtype), num_item))

    def _arg(self, cmdlist, temp_storage, d_in, d_out, d_index_out, num_item, op):
        dt = lcpp_dtype(d_in)
        pin, pout, pidx = _ptr(d_in), _ptr(d_out), _ptr(d_index_out)
        ptmp, nt = _ptr(temp_storage), _nbytes(temp_storage)
        self._record(cmdlist, lambda s: L.lib().lcpp_arg_reduce(op, dt, pin, pout, pidx, num_item, ptmp, nt, s),
                     "DeviceReduce.Arg")

    def ArgMin(self, cmdlist, temp_storage, d_in, d_out, d_index_out, num_item):
        self._arg(cmdlist, temp_storage, d_in, d_out, d_index_out, num_item, L.OP_MIN)

    def ArgMax(self, cmdlist, temp_storage, d_in, d_out, d_index_out, num_item):
        self._arg(cmdlist, temp_storage, d_in, d_out, d_index_out, num_item, L.OP_MAX)


    # ---- ReduceByKey (device_reduce.h:110-125, 277-325) ---------------------
    @staticmethod
    def GetReduceByKeyTempStorageBytes(num_elements: int, key_dtype=torch.int32, value_dtype=torch.int32) -> int:
        return int(L.lib().lcpp_reduce_by_key_temp_bytes(lcpp_dtype(key_dtype), lcpp_dtype(value_dtype),
                                                         num_elements))

    def ReduceByKey(self, cmdlist, temp_storage, d_keys_in, d_values_in, d_unique_out, g_aggregates_out,
                    g_num_runs_out, reduce_op, num_elements):
        """reduce_op: "sum" | "min" | "max" (or LCPP_OP_*); g_num_runs_out: one uint32 on the device."""
        kdt, vdt = lcpp_dtype(d_keys_in), lcpp_dtype(d_values_in)
        if lcpp_dtype(d_unique_out) != kdt or lcpp_dtype(g_aggregates_out) != vdt:
            raise TypeError("output element types must match the key / value types")
        if g_num_runs_out.dtype not in (torch.uint32, torch.int32):
            raise TypeError("g_num_runs_out must hold 32-bit unsigned integers")
        op = _op_code(reduce_op)
        pk, pv, pu, pa, pn = (_ptr(d_keys_in), _ptr(d_values_in), _ptr(d_unique_out), _ptr(g_aggregates_out),
                              _ptr(g_num_runs_out))
        ptmp, nt = _ptr(temp_storage), _nbytes(temp_storage)
        self._record(cmdlist,
                     lambda s: L.lib().lcpp_reduce_by_key(op, kdt, vdt, pk, pv, pu, pa, pn, num_elements, ptmp, nt, s),
                     "DeviceReduce.ReduceByKey")


class DeviceScan(_Module):
    @staticmethod
    def GetTempStorageBytes(num_items: int, dtype=torch.uint32) -> int:
        return int(L.lib().lcpp_scan_temp_bytes(lcpp_dtype(dtype), num_items))

    def _scan(self, kind, cmdlist, temp_storage, d_in, d_out, num_items, carry=None):
        dt = lcpp_dtype(d_in)
        if lcpp_dtype(d_out) != dt:
            raise TypeError("d_in and d_out must have the same element type")
        pin, pout, ptmp, nt, pc = _ptr(d_in), _ptr(d_out), _ptr(temp_storage), _nbytes(temp_storage), _ptr(carry)
        self._record(cmdlist,
                     lambda s: L.lib().lcpp_scan_carry(kind, dt, pin, pout, num_items, pc, ptmp, nt, s),
                     "DeviceScan")

    def ExclusiveSum(self, cmdlist, temp_storage, d_in, d_out, num_items):
        self._scan(L.SCAN_EXCLUSIVE, cmdlist, temp_storage, d_in, d_out, num_items)

    def InclusiveSum(self, cmdlist, temp_storage, d_in, d_out, num_items):
        self._scan(L.SCAN_INCLUSIVE, cmdlist, temp_storage, d_in, d_out, num_items)

    def _scan_op(self, kind, cmdlist, temp_storage, d_in, d_out, num_items, scan_op, initial_value):
        import numpy as np

        dt = lcpp_dtype(d_in)
        npdt = {L.I32: np.int32, L.U32: np.uint32, L.F32: np.float32}[dt]
        init = np.array([initial_value], dtype=npdt)
        pin, pout, ptmp, nt = _ptr(d_in), _ptr(d_out), _ptr(temp_storage), _nbytes(temp_storage)
        op = {"sum": L.OP_SUM, "min": L.OP_MIN, "max": L.OP_MAX}[scan_op] if isinstance(scan_op, str) else int(scan_op)
        self._record(cmdlist,
                     lambda s: L.lib().lcpp_scan_op(kind, op, dt, pin, pout, num_items, init.ctypes.data, ptmp, nt, s),
                     "DeviceScan")

    def ExclusiveScan(self, cmdlist, temp_storage, d_in, d_out, num_items, scan_op, initial_value):
        """scan_op: "sum" | "min" | "max" (or LCPP_OP_*), as the reference's SumOp/MinOp/MaxOp."""
        self._scan_op(L.SCAN_EXCLUSIVE, cmdlist, temp_storage, d_in, d_out, num_items, scan_op, initial_value)

    def InclusiveScan(self, cmdlist, temp_storage, d_in, d_out, num_items, scan_op, initial_value):
        self._scan_op(L.SCAN_INCLUSIVE, cmdlist, temp_storage, d_in, d_out, num_items, scan_op, initial_value)


    # ---- ScanByKey (device_scan.h:93-107, 206-345) -------------------------
    @staticmethod
    def GetScanByKeyTempStorageBytes(num_items: int, key_dtype=torch.int32, value_dtype=torch.int32) -> int:
        return int(L.lib().lcpp_scan_by_key_temp_bytes(lcpp_dtype(key_dtype), lcpp_dtype(value_dtype), num_items))

    def _scan_by_key(self, kind, cmdlist, temp_storage, d_keys_in, d_values_in, d_values_out, scan_op,
                     num_items, initial_value):
        kdt, vdt = lcpp_dtype(d_keys_in), lcpp_dtype(d_values_in)
        if lcpp_dtype(d_values_out) != vdt:
            raise TypeError("d_values_in and d_values_out must have the same element type")
        init = _host_scalar(initial_value, vdt)
        op = _op_code(scan_op)
        pk, pv, po = _ptr(d_keys_in), _ptr(d_values_in), _ptr(d_values_out)
        ptmp, nt = _ptr(temp_storage), _nbytes(temp_storage)
        self._record(cmdlist,
                     lambda s: L.lib().lcpp_scan_by_key(kind, op, kdt, vdt, pk, pv, po, num_items,
                                                        init.ctypes.data, ptmp, nt, s),
                     "DeviceScan.ScanByKey")

    def ExclusiveScanByKey(self, cmdlist, temp_storage, d_keys_in, d_values_in, d_values_out, scan_op,
                           num_items, initial_value):
        self._scan_by_key(L.SCAN_EXCLUSIVE, cmdlist, temp_storage, d_keys_in, d_values_in, d_values_out,
                          scan_op, num_items, initial_value)

    def InclusiveScanByKey(self, cmdlist, temp_storage, d_keys_in, d_values_in, d_values_out, scan_op,
                           num_items, initial_value):
        self._scan_by_key(L.SCAN_INCLUSIVE, cmdlist, temp_storage, d_keys_in, d_values_in, d_values_out,
                          scan_op, num_items, initial_value)

    def ExclusiveSumByKey(self, cmdlist, temp_storage, d_keys_in, d_values_in, d_values_out, num_items):
        self.ExclusiveScanByKey(cmdlist, temp_storage, d_keys_in, d_values_in, d_values_out, "sum", num_items, 0)

    def InclusiveSumByKey(self, cmdlist, temp_storage, d_keys_in, d_values_in, d_values_out, num_items):
        self.InclusiveScanByKey(cmdlist, temp_storage, d_keys_in, d_values_in, d_values_out, "sum", num_items, 0)


class DeviceRadixSort(_Module):
    @staticmethod
    def GetSortPairsTempStorageBytes(num_items: int, key_dtype=torch.uint32, value_dtype=torch.uint32) -> int:
        return int(L.lib().lcpp_radix_sort_temp_bytes(lcpp_dtype(key_dtype), lcpp_dtype(value_dtype), num_items))

    @staticmethod
    def GetSortKeysTempStorageBytes(num_items: int, key_dtype=torch.uint32) -> int:
        return int(L.lib().lcpp_radix_sort_temp_bytes(lcpp_dtype(key_dtype), L.NONE, num_items))

    def _sort(self, cmdlist, temp_storage, kin, kout, vin, vout, num_items, desc, begin_bit=0, end_bit=0):
        kd = lcpp_dtype(kin)
        vd = L.NONE if vin is None else lcpp_dtype(vin)
        if lcpp_dtype(kout) != kd or (vin is not None and lcpp_dtype(vout) != vd):
            raise TypeError("input and output buffers must have the same element types")
        pki, pko, pvi, pvo = _ptr(kin), _ptr(kout), _ptr(vin), _ptr(vout)
        ptmp, nt = _ptr(temp_storage), _nbytes(temp_storage)
        self._record(cmdlist,
                     lambda s: L.lib().lcpp_radix_sort(kd, vd, int(desc), pki, pko, pvi, pvo, num_items,
                                                       begin_bit, end_bit, ptmp, nt, s),
                     "DeviceRadixSort")

    def SortPairs(self, cmdlist, temp_storage, d_keys_in, d_keys_out, d_values_in, d_values_out, num_items):
        self._sort(cmdlist, temp_storage, d_keys_in, d_keys_out, d_values_in, d_values_out, num_items, False)

    def SortKeys(self, cmdlist, temp_storage, d_keys_in, d_keys_out, num_items):
        self._sort(cmdlist, temp_storage, d_keys_in, d_keys_out, None, None, num_items, False)

    def SortPairsDescending(self, cmdlist, temp_storage, d_keys_in, d_keys_out, d_values_in, d_values_out,
                            num_items):
        self._sort(cmdlist, temp_storage, d_keys_in, d_keys_out, d_values_in, d_values_out, num_items, True)

    def SortKeysDescending(self, cmdlist, temp_storage, d_keys_in, d_keys_out, num_items):
        self._sort(cmdlist, temp_storage, d_keys_in, d_keys_out, None, None, num_items, True)


class DeviceSegmentReduce(_Module):
    @staticmethod
    def GetTempStorageBytes(num_item: int, num_segments: int = 0, dtype=torch.float32) -> int:
        return int(L.lib().lcpp_segment_reduce_temp_bytes(lcpp_dtype(dtype), num_item, num_segments))

    def Reduce(self, cmdlist, temp_storage, d_in, d_out, num_segments, begin_or_size, d_end_offsets, op):
        dt = lcpp_dtype(d_in)
        pin, pout = _ptr(d_in), _ptr(d_out)
        if d_end_offsets is None:  # fixed-size overload: (num_segments, segment_size)
            size = int(begin_or_size)
            self._record(cmdlist,
                         lambda s: L.lib().lcpp_segment_reduce_fixed(op, dt, pin, pout, num_segments, size, s),
                         "DeviceSegmentReduce")
            return
        pb, pe = _ptr(begin_or_size), _ptr(d_end_offsets)
        ptmp, nt = _ptr(temp_storage), _nbytes(temp_storage)
        self._record(cmdlist,
                     lambda s: L.lib().lcpp_segment_reduce(op, dt, pin, pout, num_segments, pb, pe, ptmp, nt, s),
                     "DeviceSegmentReduce")

    def Sum(self, cmdlist, temp_storage, d_in, d_out, num_segments, d_begin_offsets_or_size, d_end_offsets=None):
        self.Reduce(cmdlist, temp_storage, d_in, d_out, num_segments, d_begin_offsets_or_size, d_end_offsets,
                    L.OP_SUM)

    def Min(self, cmdlist, temp_storage, d_in, d_out, num_segments, d_begin_offsets_or_size, d_end_offsets=None):
        self.Reduce(cmdlist, temp_storage, d_in, d_out, num_segments, d_begin_offsets_or_size, d_end_offsets,
                    L.OP_MIN)

    def Max(self, cmdlist, temp_storage, d_in, d_out, num_segments, d_begin_offsets_or_size, d_end_offsets=None):
        self.Reduce(cmdlist, temp_storage, d_in, d_out, num_segments, d_begin_offsets_or_size, d_end_offsets,
                    L.OP_MAX)


def _segment_arg(self, cmdlist, d_in, d_out, d_index_out, num_segments, begin_or_size, d_end_offsets, op):
    dt = lcpp_dtype(d_in)
    pin, pout, pidx = _ptr(d_in), _ptr(d_out), _ptr(d_index_out)
    if d_end_offsets is None:
        size = int(begin_or_size)
        self._record(cmdlist, lambda s: L.lib().lcpp_segment_arg_reduce_fixed(op, dt, pin, pout, pidx,
                                                                              num_segments, size, s),
                     "DeviceSegmentReduce.Arg")
        return
    pb, pe = _ptr(begin_or_size), _ptr(d_end_offsets)
    self._record(cmdlist, lambda s: L.lib().lcpp_segment_arg_reduce(op, dt, pin, pout, pidx, num_segments, pb, pe, s),
                 "DeviceSegmentReduce.Arg")


DeviceSegmentReduce.GetArgTempStorageBytes = staticmethod(lambda num_item, num_segments=0, dtype=None: 0)
DeviceSegmentReduce.ArgMin = lambda self, cmdlist, temp_storage, d_in, d_out, d_index_out, num_segments, b, e=None: \
    _segment_arg(self, cmdlist, d_in, d_out, d_index_out, num_segments, b, e, L.OP_MIN)
DeviceSegmentReduce.ArgMax = lambda self, cmdlist, temp_storage, d_in, d_out, d_index_out, num_segments, b, e=None: \
    _segment_arg(self, cmdlist, d_in, d_out, d_index_out, num_segments, b, e, L.OP_MAX)


def temp_buffer(nbytes: int, device="cuda") -> torch.Tensor:
    """A caller-owned temp buffer of at least nbytes (BufferView<uint> in the reference)."""
    return torch.empty(max(1, (nbytes + 3) // 4), dtype=torch.int32, device=device)


def last_device_error(stream=None) -> int:
    return int(L.lib().lcpp_last_device_error(_stream_handle(stream)))
