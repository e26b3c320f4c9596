"""ArgMin / ArgMax parity on the GPU (whole array and segments) against the
CPU oracle and the reference tests' known answers
(tests/device_reduce_test.cpp:168-220, tests/device_segment_reduce.cpp:179-293)."""
import numpy as np
import pytest

import oracle
from lc_parallel_primitive_b200 import _lib as L
from lc_parallel_primitive_b200 import datagen as G
from tests.helpers import NP2LCPP, empty_dev, refgen, stream, temp, to_dev, to_host

pytestmark = pytest.mark.gpu


def abi_arg(op, x, offset=0):
    import torch

    lib = L.lib()
    dt = NP2LCPP[x.dtype]
    d = to_dev(x, offset)
    v = empty_dev(1, x.dtype)
    i = torch.empty(1, dtype=torch.int32, device="cuda")
    tb = lib.lcpp_arg_reduce_temp_bytes(dt, x.size)
    t = temp(tb)
    L.check(lib.lcpp_arg_reduce(op, dt, d.data_ptr(), v.data_ptr(), i.data_ptr(), x.size, t.data_ptr(), tb, stream()))
    torch.cuda.synchronize()
    return to_host(v)[0], int(to_host(i).view(np.uint32)[0])


def abi_seg_arg(op, x, b, e):
    import torch

    lib = L.lib()
    dt = NP2LCPP[x.dtype]
    S = b.size
    v = empty_dev(S, x.dtype)
    i = torch.empty(S, dtype=torch.int32, device="cuda")
    db, de = to_dev(b.astype(np.uint32)), to_dev(e.astype(np.uint32))
    L.check(lib.lcpp_segment_arg_reduce(op, dt, to_dev(x).data_ptr(), v.data_ptr(), i.data_ptr(), S,
                                        db.data_ptr(), de.data_ptr(), stream()))
    torch.cuda.synchronize()
    return to_host(v), to_host(i).view(np.uint32)


def test_reference_argmin_argmax_shuffled_iota(cuda):
    g = refgen("reduce_minmax")
    x = g["input"]
    assert abi_arg(1, x) == (0, int(np.argmin(x)))
    assert abi_arg(2, x) == (4095, int(np.argmax(x)))


@pytest.mark.parametrize("dtype", [np.int32, np.uint32, np.float32, np.int64, np.float64])
def test_arg_vs_oracle_with_ties(cuda, dtype):
    for k, n in enumerate([1, 2, 33, 1000, 65537, (1 << 22) + 3]):
        raw = G.u32_below(n, 50, seed=60 + k)  # many ties
        x = raw.astype(dtype)
        for op in (1, 2):
            got = abi_arg(op, x, offset=k % 3)
            want = oracle.arg_reduce(op, x)
            assert got[1] == want[1] and got[0] == want[0], (n, op, got, want)


def test_arg_empty(cuda):
    x = np.zeros(0, dtype=np.int32)
    assert abi_arg(1, x) == (np.iinfo(np.int32).max, 1)
    assert abi_arg(2, x) == (np.iinfo(np.int32).min, 1)


def test_segment_arg_vs_oracle(cuda):
    off = G.lognormal_offsets(3000, 400000, seed=7)
    b, e = off[:-1], off[1:]
    for dtype in (np.int32, np.float32, np.uint64):
        x = G.u32_below(400000, 1000, seed=8).astype(dtype)
        for op in (1, 2):
            gv, gi = abi_seg_arg(op, x, b, e)
            wv, wi = oracle.segment_arg_reduce(op, x, b, e)
            assert np.array_equal(gv, wv) and np.array_equal(gi, wi), (dtype, op)


def test_segment_arg_fixed(cuda):
    import torch

    x = G.i32_range(32 * 1000, -100, 100, seed=9)
    v = empty_dev(1000, np.int32)
    i = torch.empty(1000, dtype=torch.int32, device="cuda")
    L.check(L.lib().lcpp_segment_arg_reduce_fixed(2, L.I32, to_dev(x).data_ptr(), v.data_ptr(), i.data_ptr(), 1000, 32,
                                                  stream()))
    torch.cuda.synchronize()
    b = (np.arange(1000) * 32).astype(np.uint32)
    wv, wi = oracle.segment_arg_reduce(2, x, b, b + 32)
    assert np.array_equal(to_host(v), wv) and np.array_equal(to_host(i).view(np.uint32), wi)
