"""TransformReduce parity on the GPU against the CPU oracle and the reference
test's known answer (tests/device_reduce_test.cpp:92-116)."""
import numpy as np
import pytest

import oracle
from tests.helpers import NP2LCPP, empty_dev, refgen, stream, temp, to_dev, to_host

pytestmark = pytest.mark.gpu

DTYPES = [np.int32, np.uint32, np.float32, np.int64, np.uint64, np.float64]
SIZES = [0, 1, 3, 4097, 100003, (1 << 22) + 7]


def abi_transform_reduce(op, xf, x, init=None, offset_elems=0):
    import torch
    from lc_parallel_primitive_b200 import _lib as L

    lib = L.lib()
    dt = NP2LCPP[x.dtype]
    d = to_dev(x, offset_elems) if x.size else empty_dev(1, x.dtype)
    out = empty_dev(1, x.dtype)
    tb = lib.lcpp_reduce_temp_bytes(dt, x.size)
    t = temp(tb)
    iv = None if init is None else np.array([init], dtype=x.dtype)
    L.check(lib.lcpp_transform_reduce(op, xf, dt, d.data_ptr(), out.data_ptr(), x.size,
                                      None if iv is None else iv.ctypes.data, t.data_ptr(), tb, stream()))
    torch.cuda.synchronize()
    return to_host(out)[0]


def test_reference_max_of_squares(cuda):
    # through the Python mirror, as the reference test calls it
    import torch
    from lc_parallel_primitive_b200 import CommandList, DeviceReduce, Stream, synchronize, temp_buffer

    g = refgen("reduce_minmax")
    reducer = DeviceReduce()
    st = Stream()
    reducer.create(None, st)
    cmdlist = CommandList()
    d_in = torch.from_numpy(g["input"]).to(cuda)
    d_out = torch.empty(1, dtype=torch.int32, device=cuda)
    tb = temp_buffer(DeviceReduce.GetTempStorageBytes(d_in.numel(), torch.int32))
    reducer.TransformReduce(cmdlist, tb, d_in, d_out, d_in.numel(), "max", "square", 0)
    st << cmdlist.commit() << synchronize()
    assert int(d_out.item()) == 4095 * 4095


@pytest.mark.parametrize("dtype", DTYPES)
def test_transform_reduce_vs_oracle(cuda, dtype):
    rng = np.random.default_rng(5)
    for i, n in enumerate(SIZES):
        if np.dtype(dtype).kind == "f":
            x = rng.standard_normal(n).astype(dtype)
        else:
            info = np.iinfo(dtype)
            x = rng.integers(info.min, info.max, size=n, dtype=dtype, endpoint=True)
        for op in (0, 1, 2):
            for xf in (0, 1, 2, 3):
                init = None if i % 2 else (3 if op == 0 else None)
                got = abi_transform_reduce(op, xf, x, init=init, offset_elems=i % 3)
                ref = oracle.transform_reduce(op, xf, x, init)
                if np.dtype(dtype).kind == "f" and op == 0:
                    scale = oracle.transform_reduce(0, 2, x.astype(np.float64) if xf != 1 else x * x) + 3
                    assert abs(float(got) - float(ref)) <= 1e-5 * float(scale) + 1e-30, (n, op, xf)
                else:
                    assert got == ref or (np.isnan(got) and np.isnan(ref)), (n, op, xf, got, ref)
