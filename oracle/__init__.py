"""CPU oracle for LCPP's device primitives — TEST INFRASTRUCTURE ONLY.

Used by tests/, __graft_entry__.smoke() (as the checker) and bench.py's
cpu_baseline / reference arm (as the timed CPU baseline).  The product path
(lc_parallel_primitive_b200) never imports this package.

Parity pinning: the reference (LuisaCompute DSL) cannot be built here; the
oracle is pinned on the reference tests' own std:: known answers, regenerated
by tests/golden/refgen.cpp (see tests/test_oracle.py).
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from .build import ORACLE_SO, build_oracle

I32, U32, F32, I64, U64, F64, NONE = 0, 1, 2, 3, 4, 5, 15
OP_SUM, OP_MIN, OP_MAX = 0, 1, 2

_NP = {np.dtype(np.int32): I32, np.dtype(np.uint32): U32, np.dtype(np.float32): F32,
       np.dtype(np.int64): I64, np.dtype(np.uint64): U64, np.dtype(np.float64): F64}

_lib = None


def lib():
    global _lib
    if _lib is None:
        if not ORACLE_SO.exists():
            build_oracle()
        h = C.CDLL(str(ORACLE_SO))
        vp, u64, i = C.c_void_p, C.c_uint64, C.c_int
        h.oracle_reduce.argtypes = [i, i, vp, u64, vp]
        h.oracle_scan.argtypes = [i, i, vp, u64, vp]
        h.oracle_abs_prefix_f32.argtypes = [vp, u64, vp]
        h.oracle_abs_prefix_f64.argtypes = [vp, u64, vp]
        h.oracle_radix_sort.argtypes = [i, i, i, vp, vp, vp, vp, u64, i, i, i]
        h.oracle_segment_reduce.argtypes = [i, i, vp, vp, u64, vp, vp]
        h.oracle_reduce_sum_mt.argtypes = [i, vp, u64, vp, i]
        h.oracle_arg_reduce.argtypes = [i, i, vp, u64, vp, vp]
        h.oracle_scan_op.argtypes = [i, i, i, vp, u64, vp, vp]
        h.oracle_segment_arg_reduce.argtypes = [i, i, vp, vp, vp, u64, vp, vp]
        h.oracle_scan_mt.argtypes = [i, i, vp, vp, u64, i]
        h.oracle_segment_reduce_mt.argtypes = [i, i, vp, vp, u64, vp, vp, i]
        h.oracle_scan_by_key.argtypes = [i, i, i, i, vp, vp, u64, vp, vp]
        h.oracle_transform_reduce.argtypes = [i, i, i, vp, u64, vp, vp]
        h.oracle_reduce_by_key.argtypes = [i, i, i, vp, vp, u64, vp, vp, vp]
        for f in ("oracle_reduce", "oracle_scan", "oracle_abs_prefix_f32", "oracle_radix_sort",
                  "oracle_segment_reduce", "oracle_reduce_sum_mt", "oracle_scan_mt",
                  "oracle_segment_reduce_mt", "oracle_arg_reduce", "oracle_segment_arg_reduce", "oracle_scan_op",
                  "oracle_scan_by_key", "oracle_reduce_by_key", "oracle_transform_reduce"):
            getattr(h, f).restype = i
        _lib = h
    return _lib


def _dt(a: np.ndarray) -> int:
    return _NP[a.dtype]


def _p(a):
    return None if a is None else a.ctypes.data


def _ok(rc, what):
    if rc != 0:
        raise ValueError(f"oracle {what} rejected its arguments")


def reduce(op: int, x: np.ndarray):
    """Integer: exact wrapped result in x.dtype.  Float: fp64 value."""
    x = np.ascontiguousarray(x)
    out = np.zeros(1, dtype=np.float64 if x.dtype.kind == "f" else x.dtype)
    _ok(lib().oracle_reduce(op, _dt(x), _p(x), x.size, _p(out)), "reduce")
    return out[0]


def scan(inclusive: bool, x: np.ndarray) -> np.ndarray:
    """Integers: exact wrapped prefixes in x.dtype.  f32: fp64 prefixes.
    f64: prefixes accumulated in long double, rounded to fp64."""
    x = np.ascontiguousarray(x)
    out = np.empty(x.size, dtype=np.float64 if x.dtype == np.float32 else x.dtype)
    _ok(lib().oracle_scan(int(inclusive), _dt(x), _p(x), x.size, _p(out)), "scan")
    return out


def abs_prefix(x: np.ndarray) -> np.ndarray:
    """Running sum of |x| in fp64 (the scale of the float-scan tolerance)."""
    if x.dtype == np.float64:
        x = np.ascontiguousarray(x)
        out = np.empty(x.size, dtype=np.float64)
        lib().oracle_abs_prefix_f64(_p(x), x.size, _p(out))
        return out
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.size, dtype=np.float64)
    lib().oracle_abs_prefix_f32(_p(x), x.size, _p(out))
    return out


def radix_sort(keys: np.ndarray, values: np.ndarray | None = None, descending=False, begin_bit=0,
               end_bit=0, threads=1):
    keys = np.ascontiguousarray(keys)
    ko = np.empty_like(keys)
    vo = None
    vd = NONE
    if values is not None:
        values = np.ascontiguousarray(values)
        vo = np.empty_like(values)
        vd = _dt(values) if values.dtype in _NP else (U32 if values.itemsize == 4 else U64)
    _ok(lib().oracle_radix_sort(_dt(keys), vd, int(descending), _p(keys), _p(ko), _p(values), _p(vo),
                                keys.size, begin_bit, end_bit, threads), "radix_sort")
    return (ko, vo) if values is not None else ko


def segment_reduce(op: int, x: np.ndarray, begin: np.ndarray, end: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x)
    begin = np.ascontiguousarray(begin, dtype=np.uint32)
    end = np.ascontiguousarray(end, dtype=np.uint32)
    out = np.empty(begin.size, dtype=np.float64 if x.dtype.kind == "f" else x.dtype)
    _ok(lib().oracle_segment_reduce(op, _dt(x), _p(x), _p(out), begin.size, _p(begin), _p(end)),
        "segment_reduce")
    return out


# ---- multi-threaded baselines (element-type arithmetic) --------------------
def reduce_sum_mt(x: np.ndarray, threads: int):
    out = np.zeros(1, dtype=x.dtype)
    _ok(lib().oracle_reduce_sum_mt(_dt(x), _p(x), x.size, _p(out), threads), "reduce_sum_mt")
    return out[0]


def scan_mt(inclusive: bool, x: np.ndarray, out: np.ndarray, threads: int):
    _ok(lib().oracle_scan_mt(int(inclusive), _dt(x), _p(x), _p(out), x.size, threads), "scan_mt")
    return out


def segment_reduce_mt(op: int, x, begin, end, out, threads: int):
    _ok(lib().oracle_segment_reduce_mt(op, _dt(x), _p(x), _p(out), begin.size, _p(begin), _p(end), threads),
        "segment_reduce_mt")
    return out


def arg_reduce(op: int, x: np.ndarray):
    """(value, index) of the min (op=OP_MIN, first index) or max (OP_MAX, last index)."""
    x = np.ascontiguousarray(x)
    v = np.zeros(1, dtype=x.dtype)
    i = np.zeros(1, dtype=np.uint32)
    _ok(lib().oracle_arg_reduce(op, _dt(x), _p(x), x.size, _p(v), _p(i)), "arg_reduce")
    return v[0], int(i[0])


def segment_arg_reduce(op: int, x: np.ndarray, begin: np.ndarray, end: np.ndarray):
    x = np.ascontiguousarray(x)
    begin = np.ascontiguousarray(begin, dtype=np.uint32)
    end = np.ascontiguousarray(end, dtype=np.uint32)
    v = np.empty(begin.size, dtype=x.dtype)
    i = np.empty(begin.size, dtype=np.uint32)
    _ok(lib().oracle_segment_arg_reduce(op, _dt(x), _p(x), _p(v), _p(i), begin.size, _p(begin), _p(end)),
        "segment_arg_reduce")
    return v, i


def scan_op(inclusive: bool, op: int, x: np.ndarray, init) -> np.ndarray:
    """Scan with SUM/MIN/MAX and an initial value, in the element type."""
    x = np.ascontiguousarray(x)
    iv = np.array([init], dtype=x.dtype)
    out = np.empty_like(x)
    _ok(lib().oracle_scan_op(int(inclusive), op, _dt(x), _p(x), x.size, _p(iv), _p(out)), "scan_op")
    return out


def _limits(dt):
    """(lowest, max) of a dtype, the identities of Max / Min."""
    dt = np.dtype(dt)
    if dt.kind == "f":
        fi = np.finfo(dt)
        return fi.min, fi.max
    ii = np.iinfo(dt)
    return ii.min, ii.max


def _out_dtype(x: np.ndarray):
    return np.dtype(np.float64) if x.dtype.kind == "f" else x.dtype


def scan_by_key(inclusive: bool, op: int, keys: np.ndarray, values: np.ndarray, init=None) -> np.ndarray:
    """Per-segment scan (segments = runs of equal keys).  Integer values: exact,
    in the value dtype.  Float values: fp64 results."""
    keys, values = np.ascontiguousarray(keys), np.ascontiguousarray(values)
    if keys.size != values.size:
        raise ValueError("keys and values differ in length")
    if init is None:
        init = {OP_SUM: 0, OP_MIN: _limits(values.dtype)[1], OP_MAX: _limits(values.dtype)[0]}[op]
    iv = np.array([init], dtype=values.dtype)
    out = np.empty(values.size, dtype=_out_dtype(values))
    _ok(lib().oracle_scan_by_key(int(inclusive), op, _dt(keys), _dt(values), _p(keys), _p(values), values.size,
                                 _p(iv), _p(out)), "scan_by_key")
    return out


def reduce_by_key(op: int, keys: np.ndarray, values: np.ndarray):
    """(unique_keys, aggregates, num_runs); float aggregates in fp64."""
    keys, values = np.ascontiguousarray(keys), np.ascontiguousarray(values)
    if keys.size != values.size:
        raise ValueError("keys and values differ in length")
    uk = np.empty(max(keys.size, 1), dtype=keys.dtype)
    agg = np.empty(max(keys.size, 1), dtype=_out_dtype(values))
    nr = np.zeros(1, dtype=np.uint32)
    _ok(lib().oracle_reduce_by_key(op, _dt(keys), _dt(values), _p(keys), _p(values), keys.size, _p(uk),
                                   _p(agg), _p(nr)), "reduce_by_key")
    r = int(nr[0])
    return uk[:r], agg[:r], r


def transform_reduce(op: int, xf: int, x: np.ndarray, init=None):
    """op(init, reduce(xf(x))); xf 0 identity, 1 square, 2 abs, 3 negate.
    Integer: exact wrapped value in x.dtype.  Float: fp64 value."""
    x = np.ascontiguousarray(x)
    if init is None:
        init = {OP_SUM: 0, OP_MIN: _limits(x.dtype)[1], OP_MAX: _limits(x.dtype)[0]}[op]
    iv = np.array([init], dtype=x.dtype)
    out = np.zeros(1, dtype=np.float64 if x.dtype.kind == "f" else x.dtype)
    _ok(lib().oracle_transform_reduce(op, xf, _dt(x), _p(x), x.size, _p(iv), _p(out)), "transform_reduce")
    return out[0]
