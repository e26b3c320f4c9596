"""DeviceSegmentReduce parity on the GPU against the CPU oracle and the
reference tests' known answers (tests/device_segment_reduce.cpp)."""
import numpy as np
import pytest

import oracle
from lc_parallel_primitive_b200 import datagen as G
from tests.helpers import abi_segment_reduce, abi_segment_reduce_fixed, refgen

pytestmark = pytest.mark.gpu


def test_reference_offsets_sum(cuda):
    # device_segment_reduce.cpp:62-125 through the Python mirror class.
    import torch
    from lc_parallel_primitive_b200 import CommandList, DeviceSegmentReduce, Stream, synchronize, temp_buffer

    g = refgen("segment_reduce")
    reducer = DeviceSegmentReduce()
    stream = Stream()
    reducer.create(None, stream)
    S = g["begin"].size
    d_in = torch.from_numpy(g["input"]).to(cuda)
    d_out = torch.empty(S, dtype=torch.int32, device=cuda)
    b = torch.from_numpy(g["begin"]).to(cuda)
    e = torch.from_numpy(g["end"]).to(cuda)
    temp = temp_buffer(DeviceSegmentReduce.GetTempStorageBytes(g["input"].size, S, torch.int32))
    cmdlist = CommandList()
    reducer.Sum(cmdlist, temp, d_in, d_out, S, b, e)
    stream << cmdlist.commit() << synchronize()
    assert np.array_equal(d_out.cpu().numpy(), g["expected"])


def test_reference_fixed_size_sum(cuda):
    # device_segment_reduce.cpp:127-176: 32 segments of 32.
    g = refgen("fixed_segment_reduce")
    assert np.array_equal(abi_segment_reduce_fixed(0, g["input"], 32, 32), g["expected"])


def _segments(S, N, seed):
    off = G.lognormal_offsets(S, N, seed=seed)
    return off[:-1], off[1:]


@pytest.mark.parametrize("op", [0, 1, 2])
@pytest.mark.parametrize("dtype", [np.int32, np.uint32, np.int64, np.uint64])
def test_integer_bit_exact(cuda, op, dtype):
    N, S = 300000, 3000
    b, e = _segments(S, N, 400 + op)
    x = (G.u32 if np.dtype(dtype).itemsize == 4 else G.u64)(N, seed=401).view(dtype)
    assert np.array_equal(abi_segment_reduce(op, x, b, e), oracle.segment_reduce(op, x, b, e))


@pytest.mark.parametrize("op", [0, 1, 2])
@pytest.mark.parametrize("dtype", [np.float32, np.float64])
def test_float(cuda, op, dtype):
    N, S = 300000, 3000
    b, e = _segments(S, N, 410 + op)
    x = G.f32_unit(N, seed=411).astype(dtype)
    got = abi_segment_reduce(op, x, b, e)
    want = oracle.segment_reduce(op, x, b, e)
    if op == 0:
        np.testing.assert_allclose(got.astype(np.float64), want, rtol=1e-5, atol=1e-30)
    else:
        empty = b == e
        assert np.array_equal(got[~empty], want[~empty].astype(dtype))
        assert np.array_equal(got[empty], want[empty].astype(dtype))


def test_long_and_empty_segments(cuda):
    # lengths 0, 1, 31, 4096, 4097 (block path), 100000 (block path), ragged.
    lens = np.array([0, 1, 31, 0, 4096, 4097, 100000, 0, 5, 65536, 7], dtype=np.uint64)
    off = np.concatenate([[0], np.cumsum(lens)]).astype(np.uint32)
    x = G.f32_unit(int(off[-1]), seed=5)
    b, e = off[:-1], off[1:]
    got = abi_segment_reduce(0, x, b, e)
    np.testing.assert_allclose(got, oracle.segment_reduce(0, x, b, e), rtol=1e-5, atol=0)
    xi = G.u32(int(off[-1]), seed=6).view(np.int32)
    assert np.array_equal(abi_segment_reduce(2, xi, b, e), oracle.segment_reduce(2, xi, b, e))


def test_without_temp_storage(cuda):
    # temp = NULL: every segment (long ones too) is reduced by one warp.
    lens = np.array([0, 3, 5000, 0, 70000, 1, 4096, 4097], dtype=np.uint64)
    off = np.concatenate([[0], np.cumsum(lens)]).astype(np.uint32)
    b, e = off[:-1], off[1:]
    xi = G.u32(int(off[-1]), seed=8).view(np.int32)
    for op in (0, 1, 2):
        assert np.array_equal(abi_segment_reduce(op, xi, b, e, with_temp=False), oracle.segment_reduce(op, xi, b, e))


def test_fixed_size_paths(cuda):
    for seg, S in ((1, 1000), (32, 1000), (100, 777), (4096, 50), (5000, 40), (70000, 3)):
        x = G.u32(seg * S, seed=seg).view(np.int32)
        b = np.arange(S, dtype=np.uint64) * seg
        want = oracle.segment_reduce(0, x, b.astype(np.uint32), (b + seg).astype(np.uint32))
        assert np.array_equal(abi_segment_reduce_fixed(0, x, S, seg), want), seg


def test_config4_full_size(cuda):
    # 2^27 f32 U(0,1), 2^20 lognormal(4,1.5) segments, 2 % empty.
    N, S = 1 << 27, 1 << 20
    off = G.lognormal_offsets(S, N, seed=1, stream=9)
    b, e = off[:-1], off[1:]
    x = G.f32_unit(N, seed=1, stream=10)
    got = abi_segment_reduce(0, x, b, e)
    np.testing.assert_allclose(got.astype(np.float64), oracle.segment_reduce(0, x, b, e), rtol=1e-5, atol=0)
    xi = G.u32(N, seed=1, stream=11).view(np.int32)
    got = abi_segment_reduce(2, xi, b, e)
    want = oracle.segment_reduce(2, xi, b, e)
    assert np.array_equal(got, want)
    assert (got[b == e] == np.iinfo(np.int32).min).all()
