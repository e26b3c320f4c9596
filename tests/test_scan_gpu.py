"""DeviceScan parity on the GPU against the CPU oracle and the reference tests'
known answers (tests/device_scan_test.cpp)."""
import numpy as np
import pytest

import oracle
from lc_parallel_primitive_b200 import datagen as G
from lc_parallel_primitive_b200 import _lib as L
from tests.helpers import NP2LCPP, abi_scan, assert_float_sum_close, stream, to_dev, to_host

pytestmark = pytest.mark.gpu


def test_reference_scan_of_ones(cuda):
    # tests/device_scan_test.cpp:67-108: uint Exclusive/InclusiveSum of all
    # ones, n = 2^0 .. 2^23, compared with std::exclusive_scan/inclusive_scan.
    import torch
    from lc_parallel_primitive_b200 import CommandList, DeviceScan, Stream, synchronize, temp_buffer

    scanner = DeviceScan(256, 32, 4)
    stream = Stream()
    scanner.create(None, stream)
    cmdlist = CommandList()
    for i in range(24):
        n = 1 << i
        d_in = torch.ones(n, dtype=torch.int32, device=cuda).view(torch.uint32)
        ex = torch.empty(n, dtype=torch.uint32, device=cuda)
        inc = torch.empty(n, dtype=torch.uint32, device=cuda)
        temp = temp_buffer(DeviceScan.GetTempStorageBytes(n, torch.uint32))
        scanner.ExclusiveSum(cmdlist, temp, d_in, ex, n)
        stream << cmdlist.commit() << synchronize()
        scanner.InclusiveSum(cmdlist, temp, d_in, inc, n)
        stream << cmdlist.commit() << synchronize()
        iota = np.arange(n, dtype=np.uint32)
        assert np.array_equal(to_host(ex), iota), n
        assert np.array_equal(to_host(inc), iota + 1), n


SIZES = [1, 2, 31, 32, 33, 1023, 1024, 1025, 8191, 8192, 8193, 3 * 8192 + 17, 100000, (1 << 20) + 1]


@pytest.mark.parametrize("inclusive", [False, True])
@pytest.mark.parametrize("dtype", [np.uint32, np.int32])
def test_integer_scan_bit_exact(cuda, inclusive, dtype):
    for i, n in enumerate(SIZES):
        x = G.u32(n, seed=100 + i).view(dtype)  # full range: exercises wraparound
        got = abi_scan(inclusive, x, offset_elems=i % 3)
        assert np.array_equal(got, oracle.scan(inclusive, x)), n


@pytest.mark.parametrize("inclusive", [False, True])
def test_float_scan_tolerance(cuda, inclusive):
    for i, n in enumerate(SIZES):
        x = G.f32_normal(n, seed=200 + i)
        got = abi_scan(inclusive, x, offset_elems=i % 2)
        assert_float_sum_close(got, oracle.scan(inclusive, x), oracle.abs_prefix(x))


@pytest.mark.parametrize("inclusive", [False, True])
@pytest.mark.parametrize("dtype", [np.uint64, np.int64])
def test_integer_scan_8byte_bit_exact(cuda, inclusive, dtype):
    # The reference's NumericT scans (device_scan.h:180-204) admit 8-byte types.
    for i, n in enumerate(SIZES + [3 * 4096 + 5, 4096, 16384 + 1]):
        x = G.u64(n, seed=150 + i).view(dtype)  # full range: exercises wraparound
        got = abi_scan(inclusive, x, offset_elems=i % 3)
        assert np.array_equal(got, oracle.scan(inclusive, x)), n


@pytest.mark.parametrize("inclusive", [False, True])
def test_double_scan_tolerance(cuda, inclusive):
    for i, n in enumerate(SIZES):
        x = G.f32_normal(n, seed=250 + i).astype(np.float64) * np.float64(1.0 + 1e-9)
        got = abi_scan(inclusive, x, offset_elems=i % 2)
        assert_float_sum_close(got, oracle.scan(inclusive, x), oracle.abs_prefix(x), rel=1e-12)


@pytest.mark.parametrize("dtype", [np.uint32, np.uint64, np.float64])
def test_temp_reused_across_calls(cuda, dtype):
    """A temp buffer left with another call's published descriptors (and one
    filled with 0xff bytes) must give the same results: each call clears every
    descriptor it reads."""
    import torch

    lib = L.lib()
    n = 5 * 8192 + 77
    dt = NP2LCPP[np.dtype(dtype)]
    tb = lib.lcpp_scan_temp_bytes(dt, n)
    t = torch.full((tb,), 0xFF, dtype=torch.uint8, device="cuda")
    for seed in (401, 402, 403):
        x = G.u64(n, seed=seed).view(np.uint64)
        x = (x % 1000).astype(dtype) if dtype != np.uint32 else G.u32(n, seed=seed)
        for off in (0, 1):
            d = to_dev(x, off)
            out = torch.empty_like(d)
            L.check(lib.lcpp_scan(0, dt, d.data_ptr(), out.data_ptr(), n, t.data_ptr(), tb, stream()))
            torch.cuda.synchronize()
            L.check(lib.lcpp_last_device_error(stream()))
            got = out.cpu().numpy().view(np.dtype(dtype))
            want = oracle.scan(False, x)
            if dtype == np.float64:
                np.testing.assert_allclose(got, want, rtol=1e-12, atol=1e-9)
            else:
                assert np.array_equal(got, want), (seed, off)


def test_8byte_scan_full_size(cuda):
    # 2^27 uint64 (1 GiB): bit-exact against the oracle.
    x = G.u64(1 << 27, seed=3)
    assert np.array_equal(abi_scan(False, x), oracle.scan(False, x))


def test_in_place(cuda):
    x = G.u32_below(123457, 16, seed=7)
    got = abi_scan(False, x, in_place=True)
    assert np.array_equal(got, oracle.scan(False, x))


def test_config2_exclusive_u32_full(cuda):
    # 2^28 uint32 uniform in [0,16), bit-exact.
    x = G.u32_below(1 << 28, 16, seed=1, stream=5)
    got = abi_scan(False, x)
    assert np.array_equal(got, oracle.scan(False, x))


def test_config2_inclusive_f32_full(cuda):
    # 2^28 float32 N(0,1); |y-ref| <= 1e-5*max(|ref|, sum|x|*2^-6).
    x = G.f32_normal(1 << 28, seed=1, stream=5)
    got = abi_scan(True, x)
    assert_float_sum_close(got, oracle.scan(True, x), oracle.abs_prefix(x))


@pytest.mark.parametrize("inclusive", [False, True])
@pytest.mark.parametrize("op", [1, 2])
@pytest.mark.parametrize("dtype", [np.int32, np.uint32, np.float32])
def test_min_max_scan_with_init(cuda, inclusive, op, dtype):
    # DeviceScan::ExclusiveScan / InclusiveScan with MinOp / MaxOp and an initial value.
    import torch
    from lc_parallel_primitive_b200 import _lib as L
    from tests.helpers import NP2LCPP, empty_dev, stream, temp, to_dev

    lib = L.lib()
    for k, n in enumerate([1, 1000, 8193, 100003, (1 << 21) + 5]):
        x = G.u32(n, seed=500 + k).view(np.int32).astype(dtype) if dtype != np.uint32 else G.u32(n, seed=500 + k)
        init = np.array([x[n // 2]], dtype=dtype)  # a value inside the range
        dt = NP2LCPP[np.dtype(dtype)]
        d = to_dev(x, k % 2)
        out = empty_dev(n, dtype, k % 2)
        tb = lib.lcpp_scan_temp_bytes(dt, n)
        t = temp(tb)
        L.check(lib.lcpp_scan_op(int(inclusive), op, dt, d.data_ptr(), out.data_ptr(), n, init.ctypes.data,
                                 t.data_ptr(), tb, stream()))
        torch.cuda.synchronize()
        assert np.array_equal(out.cpu().numpy(), oracle.scan_op(inclusive, op, x, init[0])), n


def test_sum_scan_with_init(cuda):
    import torch
    from lc_parallel_primitive_b200 import _lib as L
    from tests.helpers import empty_dev, stream, temp, to_dev

    lib = L.lib()
    x = G.u32(300007, seed=77)
    init = np.array([123456789], dtype=np.uint32)
    for inclusive in (False, True):
        d, out = to_dev(x), empty_dev(x.size, np.uint32)
        tb = lib.lcpp_scan_temp_bytes(L.U32, x.size)
        t = temp(tb)
        L.check(lib.lcpp_scan_op(int(inclusive), 0, L.U32, d.data_ptr(), out.data_ptr(), x.size, init.ctypes.data,
                                 t.data_ptr(), tb, stream()))
        torch.cuda.synchronize()
        assert np.array_equal(out.cpu().numpy(), oracle.scan_op(inclusive, 0, x, init[0]))
