"""lc_parallel_primitive_b200 — B200 (sm_100a) device primitives with LCPP's API.

Native code: liblcpp_b200.so (CUDA kernels + C ABI, include/lcpp_b200.h).
Python host mirror of the reference's Device* classes: primitives.py.
"""
from ._lib import LcppError, check, lib  # noqa: F401
from .primitives import (  # noqa: F401
    CommandList,
    DeviceRadixSort,
    DeviceReduce,
    DeviceScan,
    DeviceSegmentReduce,
    Stream,
    last_device_error,
    synchronize,
    temp_buffer,
)
