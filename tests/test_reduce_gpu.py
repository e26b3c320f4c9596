"""DeviceReduce parity on the GPU (through the C ABI and the Python mirror of
the reference's DeviceReduce), against the CPU oracle and the reference
tests' known answers (tests/device_reduce_test.cpp)."""
import numpy as np
import pytest

import oracle
from lc_parallel_primitive_b200 import datagen as G
from tests.helpers import abi_reduce, refgen, to_dev, to_host

pytestmark = pytest.mark.gpu


def test_reference_sum_of_ones(cuda):
    # tests/device_reduce_test.cpp:66-90: uint Sum of all-ones, n = 2^k + 1.
    import torch
    from lc_parallel_primitive_b200 import CommandList, DeviceReduce, Stream, synchronize, temp_buffer

    reducer = DeviceReduce()
    stream = Stream()
    reducer.create(None, stream)
    for loop in range(24):
        n = (1 << loop) + 1
        d_in = torch.ones(n, dtype=torch.int32, device=cuda).view(torch.uint32)
        d_out = torch.empty(1, dtype=torch.uint32, device=cuda)
        temp = temp_buffer(DeviceReduce.GetTempStorageBytes(n, torch.uint32))
        cmdlist = CommandList()
        reducer.Sum(cmdlist, temp, d_in, d_out, n)
        stream << cmdlist.commit() << synchronize()
        assert int(to_host(d_out)[0]) == n


def test_reference_min_max_shuffled_iota(cuda):
    # tests/device_reduce_test.cpp:118-166: int Min / Max of shuffled iota(4096).
    g = refgen("reduce_minmax")
    assert abi_reduce(oracle.OP_MIN, g["input"]) == g["min"][0] == 0
    assert abi_reduce(oracle.OP_MAX, g["input"]) == g["max"][0] == 4095


SIZES = [0, 1, 2, 3, 31, 32, 33, 1023, 1024, 1025, 8191, 65537, 1 << 20, (1 << 22) + 5]


@pytest.mark.parametrize("dtype", [np.int32, np.uint32, np.int64, np.uint64])
@pytest.mark.parametrize("op", [0, 1, 2])
def test_integer_reduce_bit_exact(cuda, dtype, op):
    for i, n in enumerate(SIZES):
        if np.dtype(dtype).itemsize == 4:
            x = G.u32(n, seed=10 + i).view(dtype)
        else:
            x = G.u64(n, seed=10 + i).view(dtype)
        got = abi_reduce(op, x, offset_elems=i % 3)
        want = oracle.reduce(op, x)
        assert got == want, (n, op, got, want)


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
@pytest.mark.parametrize("op", [0, 1, 2])
def test_float_reduce(cuda, dtype, op):
    for i, n in enumerate(SIZES):
        x = G.f32_normal(n, seed=20 + i).astype(dtype)
        got = abi_reduce(op, x, offset_elems=i % 2)
        want = oracle.reduce(op, x)
        if op == 0:
            # fp32/fp64 sum within 1e-5 of the fp64 oracle, relative to sum|x|
            tol = 1e-5 * max(float(np.abs(x.astype(np.float64)).sum()), 1e-30)
            assert abs(float(got) - float(want)) <= tol, (n, got, want)
        else:
            assert float(got) == float(want), (n, op, got, want)


def test_empty_gives_init(cuda):
    x = np.zeros(0, dtype=np.float32)
    assert abi_reduce(2, x) == np.float32(-3.40282347e38)  # Max of nothing: lowest()
    assert abi_reduce(1, np.zeros(0, dtype=np.int32)) == np.iinfo(np.int32).max
    assert abi_reduce(0, np.zeros(0, dtype=np.uint32)) == 0


def test_max_of_negative_floats(cuda):
    # Max starts from lowest(), not numeric_limits<float>::min() (device_reduce.h:184).
    x = -np.abs(G.f32_normal(5000, seed=3)) - 1.0
    assert abi_reduce(2, x) == x.max()


def test_config1_full_size(cuda):
    # n = 2^24 int32 uniform in [-1000, 1000], seeded PCG.
    x = G.i32_range(1 << 24, -1000, 1000, seed=1, stream=3)
    assert abi_reduce(0, x) == oracle.reduce(0, x)


def test_repeated_calls_reuse_temp(cuda):
    import torch
    from lc_parallel_primitive_b200 import _lib as L
    from tests.helpers import stream, temp

    lib = L.lib()
    x = G.u32((1 << 21) + 3, seed=5)
    d = to_dev(x)
    out = torch.empty(1, dtype=torch.uint32, device=cuda)
    tb = lib.lcpp_reduce_temp_bytes(L.U32, x.size)
    t = temp(tb)
    for _ in range(5):
        L.check(lib.lcpp_reduce(0, L.U32, d.data_ptr(), out.data_ptr(), x.size, t.data_ptr(), tb, stream()))
    torch.cuda.synchronize()
    assert to_host(out)[0] == oracle.reduce(0, x)
