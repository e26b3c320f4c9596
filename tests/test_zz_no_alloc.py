"""lcpp_scan_noalloc: the scan for callers that cannot allocate device memory
at call time (allocator callbacks, plug-ins given only their buffers,
real-time paths).  Its scratch lives in a fixed array inside the library, so
the test checks it against the regular lcpp_scan, through the C ABI, on two
calls in a row (the second call must not see the first call's leftovers).
Collected last on purpose."""
import numpy as np
import pytest

from lc_parallel_primitive_b200 import _lib as L
from lc_parallel_primitive_b200 import datagen as G
from tests.helpers import abi_scan, assert_float_sum_close, empty_dev, stream, to_dev, to_host

pytestmark = pytest.mark.gpu


def _noalloc(kind, x, offset_elems=0, in_place=False):
    import torch

    lib = L.lib()
    d = to_dev(x, offset_elems)
    out = d if in_place else empty_dev(x.size, x.dtype, offset_elems)
    dt = {np.dtype(np.uint32): L.U32, np.dtype(np.int32): L.I32, np.dtype(np.float32): L.F32}[x.dtype]
    L.check(lib.lcpp_scan_noalloc(kind, dt, d.data_ptr(), out.data_ptr(), x.size, stream()))
    torch.cuda.synchronize()
    L.check(lib.lcpp_last_device_error(stream()))
    return to_host(out)


def test_noalloc_scan_matches_regular_scan(cuda):
    # two calls in a row, different sizes and kinds
    x1 = G.u32_below((1 << 22) + 77, 16, seed=41)
    x2 = G.u32_below(300001, 1 << 20, seed=42)
    assert np.array_equal(_noalloc(0, x1), abi_scan(False, x1))
    assert np.array_equal(_noalloc(1, x2), abi_scan(True, x2))
    f = G.f32_normal(1000003, seed=43)
    got = _noalloc(1, f)
    ref = abi_scan(True, f)
    # same kernel and tile shape: within the scan tests' float tolerance
    import oracle

    assert_float_sum_close(got, ref.astype(np.float64), oracle.abs_prefix(f))


def test_noalloc_allocates_nothing_and_serves_odd_buffers(cuda):
    # Warm call first (module and array already resident), then device memory
    # in use must not change across further calls; unaligned and in-place
    # buffers take the tile kernel's scalar path.
    import torch

    x = G.u32_below(777777, 1 << 12, seed=44)
    want = abi_scan(False, x)
    assert np.array_equal(_noalloc(0, x), want)
    d = to_dev(x, 1)
    out = empty_dev(x.size, x.dtype, 3)
    lib = L.lib()
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        L.check(lib.lcpp_scan_noalloc(0, L.U32, d.data_ptr(), out.data_ptr(), x.size, stream()))
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, (free0, free1)
    assert np.array_equal(to_host(out), want)
    assert np.array_equal(_noalloc(0, x, in_place=True), want)
    assert np.array_equal(_noalloc(1, x, offset_elems=2), abi_scan(True, x))


def test_noalloc_rejects_oversize(cuda):
    lib = L.lib()
    mx = lib.lcpp_scan_noalloc_max_items()
    assert mx == 1 << 29
    assert lib.lcpp_scan_noalloc(0, L.U32, 16, 16, mx + 1, None) == L.ERR_INVALID_ARG
