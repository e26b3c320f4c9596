"""Seeded synthetic inputs (PCG32, see csrc/datagen.c) as numpy arrays.

Shapes and distributions of the benchmark configurations:
  reduce  : int32 uniform in [-1000, 1000]
  scan    : uint32 uniform in [0, 16); float32 N(0, 1)
  sort    : uint32 uniform over 2^32 (skewed: & 0xFF); values uint32 iota
  segment : float32 U[0,1) / int32 full range; lognormal(4, 1.5) lengths,
            2 % empty, scaled to sum to N
  mg sort : uint64 uniform over 2^64
"""
from __future__ import annotations

import numpy as np

from ._lib import datagen

GEN_U32, GEN_I32_RANGE, GEN_U32_BOUND, GEN_F32_NORMAL, GEN_F32_UNIT, GEN_U64, GEN_U32_MASK = range(7)


def _fill(kind, dtype, n, seed, stream, a=0, b=0, threads=0, out=None):
    arr = np.empty(n, dtype=dtype) if out is None else out
    assert arr.dtype == np.dtype(dtype) and arr.size == n and arr.flags.c_contiguous
    rc = datagen().pcg_fill(kind, arr.ctypes.data, n, seed, stream, a, b, threads)
    if rc != 0:
        raise ValueError("pcg_fill failed")
    return arr


def u32(n, seed=1, stream=0, out=None):
    return _fill(GEN_U32, np.uint32, n, seed, stream, out=out)


def u32_masked(n, mask, seed=1, stream=0, out=None):
    return _fill(GEN_U32_MASK, np.uint32, n, seed, stream, a=mask, out=out)


def i32_range(n, lo, hi, seed=1, stream=0, out=None):
    return _fill(GEN_I32_RANGE, np.int32, n, seed, stream, a=lo, b=hi, out=out)


def u32_below(n, bound, seed=1, stream=0, out=None):
    return _fill(GEN_U32_BOUND, np.uint32, n, seed, stream, a=bound, out=out)


def f32_normal(n, seed=1, stream=0, out=None):
    return _fill(GEN_F32_NORMAL, np.float32, n, seed, stream, out=out)


def f32_unit(n, seed=1, stream=0, out=None):
    return _fill(GEN_F32_UNIT, np.float32, n, seed, stream, out=out)


def u64(n, seed=1, stream=0, out=None):
    return _fill(GEN_U64, np.uint64, n, seed, stream, out=out)


def iota_u32(n, start=0, out=None):
    arr = np.empty(n, dtype=np.uint32) if out is None else out
    datagen().fill_iota_u32(arr.ctypes.data, n, start)
    return arr


def lognormal_offsets(num_segments, num_items, mu=4.0, sigma=1.5, p_empty=0.02, seed=1, stream=0):
    """CSR offsets[S+1] (uint32) whose segment lengths follow the benchmark's
    lognormal distribution and sum to exactly num_items."""
    off = np.empty(num_segments + 1, dtype=np.uint32)
    rc = datagen().pcg_segments_lognormal(off.ctypes.data, num_segments, num_items, mu, sigma, p_empty,
                                          seed, stream)
    if rc != 0:
        raise ValueError("pcg_segments_lognormal failed")
    return off
