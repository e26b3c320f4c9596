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


def _abi_seg_custom(op, x, b, e, temp_items=None, offset_elems=0):
    """lcpp_segment_reduce with the temp of lcpp_segment_reduce_temp_bytes(temp_items)
    (default: the real item count) and, optionally, an unaligned input view."""
    import torch

    from lc_parallel_primitive_b200 import _lib as L
    from tests.helpers import NP2LCPP, empty_dev, stream, temp, to_dev, to_host

    lib = L.lib()
    dt = NP2LCPP[x.dtype]
    d = to_dev(x, offset_elems)
    db, de = to_dev(b.astype(np.uint32)), to_dev(e.astype(np.uint32))
    out = empty_dev(b.size, x.dtype)
    tb = lib.lcpp_segment_reduce_temp_bytes(dt, x.size if temp_items is None else temp_items, b.size)
    t = temp(tb)
    L.check(lib.lcpp_segment_reduce(op, dt, d.data_ptr(), out.data_ptr(), b.size, db.data_ptr(), de.data_ptr(),
                                    t.data_ptr(), tb, stream()))
    torch.cuda.synchronize()
    L.check(lib.lcpp_last_device_error(stream()))
    return to_host(out)


def test_flat_path_offsets_that_are_not_csr(cuda):
    N = 200003
    xi = G.u32(N, seed=21).view(np.int32)
    rng = np.random.default_rng(21)
    # gaps between segments and a first segment that does not start at 0
    cuts = np.sort(rng.choice(np.arange(1, N), size=2 * 999, replace=False)).astype(np.uint32)
    b, e = cuts[0::2], cuts[1::2]
    for op in (0, 1, 2):
        assert np.array_equal(_abi_seg_custom(op, xi, b, e), oracle.segment_reduce(op, xi, b, e))
    # overlapping and unordered segments: the device check sends them to the per-segment kernel
    b2 = rng.integers(0, N - 5000, size=777).astype(np.uint32)
    e2 = (b2 + rng.integers(0, 5000, size=777)).astype(np.uint32)
    for op in (0, 2):
        assert np.array_equal(_abi_seg_custom(op, xi, b2, e2), oracle.segment_reduce(op, xi, b2, e2))


def test_flat_path_edges(cuda):
    xi = G.u32(1 << 20, seed=22).view(np.int32)
    # all segments empty (no tiles): every output is init
    z = np.zeros(1000, dtype=np.uint32)
    assert np.array_equal(_abi_seg_custom(2, xi[:0], z, z), np.full(1000, np.iinfo(np.int32).min, np.int32))
    # one segment over many tiles, with empty segments around it, and an exact tile edge
    TI = 8192
    lens = np.array([0, 5 * TI + 17, 0, 0, TI - 17, TI, 1, 0, 3 * TI], dtype=np.uint64)
    off = np.concatenate([[0], np.cumsum(lens)]).astype(np.uint32)
    x = xi[: int(off[-1])]
    b, e = off[:-1], off[1:]
    for op in (0, 1, 2):
        assert np.array_equal(_abi_seg_custom(op, x, b, e), oracle.segment_reduce(op, x, b, e))
    # temp sized for fewer items than the offsets reach: the device check falls back
    assert np.array_equal(_abi_seg_custom(0, x, b, e, temp_items=1), oracle.segment_reduce(0, x, b, e))
    # an input that is not 16-byte aligned (scalar tile loads)
    xf = G.f32_unit(int(off[-1]), seed=23)
    got = _abi_seg_custom(0, xf, b, e, offset_elems=1)
    np.testing.assert_allclose(got.astype(np.float64), oracle.segment_reduce(0, xf, b, e), rtol=1e-5, atol=0)
    # 8-byte values (4096-item tiles)
    x8 = G.u64(int(off[-1]), seed=24).view(np.int64)
    assert np.array_equal(_abi_seg_custom(0, x8, b, e), oracle.segment_reduce(0, x8, b, e))


@pytest.mark.gpu
def test_item_parallel_tiles(cuda):
    """Contiguous offsets: tiles of short segments (item-parallel path), heads on
    32-item thread boundaries and at tile starts, empty runs, and tiles with more
    than 511 segments (per-segment path) in one input."""
    rng = np.random.default_rng(31)
    TI = 8192
    a = rng.integers(0, 41, size=3000)                       # ~400 segments per tile
    a = np.concatenate([a, [TI - int(a.sum()) % TI]])         # the next segment starts a tile
    parts = [a,
             np.full(600, 32),                                # heads on thread boundaries
             np.array([TI - (600 * 32) % TI, 0, 0, TI]),      # heads at tile starts, empty runs
             rng.integers(0, 2, size=3000),                   # > 511 segments per tile
             rng.integers(1, 3000, size=300)]                 # long pieces crossing tiles
    lens = np.concatenate(parts).astype(np.uint64)
    off = np.concatenate([[0], np.cumsum(lens)]).astype(np.uint32)
    b, e = off[:-1], off[1:]
    xi = G.u32(int(off[-1]), seed=32).view(np.int32)
    for op in (0, 1, 2):
        assert np.array_equal(_abi_seg_custom(op, xi, b, e), oracle.segment_reduce(op, xi, b, e))
    xf = G.f32_unit(int(off[-1]), seed=33)
    np.testing.assert_allclose(_abi_seg_custom(0, xf, b, e).astype(np.float64), oracle.segment_reduce(0, xf, b, e),
                               rtol=1e-5, atol=0)
    x8 = G.u64(int(off[-1]), seed=34).view(np.int64)
    assert np.array_equal(_abi_seg_custom(2, x8, b, e), oracle.segment_reduce(2, x8, b, e))
