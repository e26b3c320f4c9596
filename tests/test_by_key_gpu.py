"""ScanByKey / ReduceByKey parity on the GPU against the CPU oracle and the
reference tests' known answers (tests/device_scan_test.cpp:111-167,
tests/device_reduce_test.cpp:229-295)."""
import numpy as np
import pytest

import oracle
from tests.helpers import abi_reduce_by_key, abi_scan_by_key, assert_float_sum_close, refgen, to_host

pytestmark = pytest.mark.gpu

KEY_DTYPES = [np.int32, np.uint32, np.float32, np.int64, np.uint64, np.float64]
VALUE_DTYPES = [np.int32, np.uint32, np.float32, np.int64, np.uint64, np.float64]
# tile = 8192 items (4-byte key and value) or 4096 (any 8-byte type)
SIZES = [1, 2, 31, 4095, 4096, 4097, 8191, 8192, 8193, 3 * 8192 + 17, 100003, (1 << 20) + 5]


def run_keys(n, mean_run, dtype, seed):
    """Keys with runs of geometric length (mean mean_run); values of a run are
    equal, consecutive runs differ."""
    rng = np.random.default_rng(seed)
    heads = rng.random(n) < 1.0 / mean_run
    ids = np.cumsum(heads)
    if np.dtype(dtype).kind == "f":
        return (ids * 0.5 - 7.25).astype(dtype)
    return (ids * 3 + 11).astype(dtype)


def values_of(n, dtype, seed):
    rng = np.random.default_rng(seed)
    if np.dtype(dtype).kind == "f":
        return rng.standard_normal(n).astype(dtype)
    info = np.iinfo(dtype)
    return rng.integers(info.min, info.max, size=n, dtype=dtype, endpoint=True)


def check_scan(got, keys, vals, inclusive, op, init):
    ref = oracle.scan_by_key(inclusive, op, keys, vals, init)
    if np.dtype(vals.dtype).kind == "f" and op == 0:
        absv = np.abs(vals)
        scale = oracle.scan_by_key(True, 0, keys, absv) + abs(float(init or 0))
        assert_float_sum_close(got, ref, scale)
    else:
        assert np.array_equal(got.astype(ref.dtype), ref)


def test_reference_exclusive_sum_by_key(cuda):
    # device_scan_test.cpp:111-167: int keys i/100, values 1, n = 2^5 .. 2^23,
    # through the Python mirror of DeviceScan::ExclusiveSumByKey.
    import torch
    from lc_parallel_primitive_b200 import CommandList, DeviceScan, Stream, synchronize, temp_buffer

    scanner = DeviceScan()
    stream = Stream()
    scanner.create(None, stream)
    cmdlist = CommandList()
    for i in range(5, 24, 3):
        n = 1 << i
        g = refgen("exclusive_sum_by_key", n)
        keys = torch.from_numpy(g["keys"]).to(cuda)
        vals = torch.from_numpy(g["values"]).to(cuda)
        out = torch.empty(n, dtype=torch.int32, device=cuda)
        temp = temp_buffer(DeviceScan.GetScanByKeyTempStorageBytes(n, torch.int32, torch.int32))
        scanner.ExclusiveSumByKey(cmdlist, temp, keys, vals, out, n)
        stream << cmdlist.commit() << synchronize()
        assert np.array_equal(to_host(out), g["expected"]), n


def test_reference_reduce_by_key(cuda):
    # device_reduce_test.cpp:229-295 through the Python mirror of ReduceByKey.
    import torch
    from lc_parallel_primitive_b200 import CommandList, DeviceReduce, Stream, synchronize, temp_buffer

    g = refgen("reduce_by_key")
    n = g["keys"].size
    reducer = DeviceReduce()
    stream = Stream()
    reducer.create(None, stream)
    cmdlist = CommandList()
    keys = torch.from_numpy(g["keys"]).to(cuda)
    vals = torch.from_numpy(g["values"]).to(cuda)
    S = g["num_runs_expected"][0]
    uk = torch.empty(S, dtype=torch.int32, device=cuda)
    agg = torch.empty(S, dtype=torch.int32, device=cuda)
    nr = torch.empty(1, dtype=torch.uint32, device=cuda)
    temp = temp_buffer(DeviceReduce.GetReduceByKeyTempStorageBytes(n, torch.int32, torch.int32))
    reducer.ReduceByKey(cmdlist, temp, keys, vals, uk, agg, nr, "sum", n)
    stream << cmdlist.commit() << synchronize()
    assert int(nr.cpu().numpy()[0]) == S
    assert np.array_equal(to_host(uk), g["unique_expected"])
    assert np.array_equal(to_host(agg), g["aggregates_expected"])


@pytest.mark.parametrize("inclusive", [False, True])
@pytest.mark.parametrize("op", [0, 1, 2])
def test_scan_by_key_u32_i32(cuda, inclusive, op):
    for i, n in enumerate(SIZES):
        for mean_run in (1.5, 37, 20000):
            keys = run_keys(n, mean_run, np.uint32, seed=i)
            vals = values_of(n, np.int32, seed=1000 + i)
            init = [5, -3, 17][i % 3]
            got = abi_scan_by_key(inclusive, op, keys, vals, init=init, offset_elems=i % 2)
            check_scan(got, keys, vals, inclusive, op, init)


@pytest.mark.parametrize("kdt", KEY_DTYPES)
@pytest.mark.parametrize("vdt", VALUE_DTYPES)
def test_scan_by_key_dtypes(cuda, kdt, vdt):
    for j, n in enumerate((4097, 70001)):
        keys = run_keys(n, 9, kdt, seed=j)
        vals = values_of(n, vdt, seed=50 + j)
        for inclusive in (False, True):
            for op in (0, 1, 2):
                got = abi_scan_by_key(inclusive, op, keys, vals)
                check_scan(got, keys, vals, inclusive, op, None)


@pytest.mark.parametrize("vdt", [np.int32, np.int64, np.float64])
def test_scan_by_key_temp_reused(cuda, vdt):
    """One temp buffer, first filled with 0xff bytes, then left with each
    call's published descriptors, serves the next calls: every call clears the
    descriptors it reads."""
    import torch

    from lc_parallel_primitive_b200 import _lib as L
    from tests.helpers import NP2LCPP

    n = 7 * 4096 + 333
    tb = L.lib().lcpp_scan_by_key_temp_bytes(NP2LCPP[np.dtype(np.int32)], NP2LCPP[np.dtype(vdt)], n)
    t = torch.full((tb,), 0xFF, dtype=torch.uint8, device="cuda")
    for j in range(3):
        keys = run_keys(n, 7 + j, np.int32, seed=300 + j)
        vals = values_of(n, vdt, seed=310 + j)
        for off in (0, 1):
            got = abi_scan_by_key(False, 0, keys, vals, offset_elems=off, temp_buf=t)
            check_scan(got, keys, vals, False, 0, None)


@pytest.mark.parametrize("kdt", KEY_DTYPES)
@pytest.mark.parametrize("vdt", VALUE_DTYPES)
def test_reduce_by_key_dtypes(cuda, kdt, vdt):
    for j, n in enumerate((1, 4097, 70001)):
        keys = run_keys(n, 5, kdt, seed=j)
        vals = values_of(n, vdt, seed=60 + j)
        for op in (0, 1, 2):
            uk, agg, r = abi_reduce_by_key(op, keys, vals)
            ruk, ragg, rr = oracle.reduce_by_key(op, keys, vals)
            assert r == rr
            assert np.array_equal(uk, ruk)
            if np.dtype(vdt).kind == "f" and op == 0:
                _, sabs, _ = oracle.reduce_by_key(0, keys, np.abs(vals))
                assert_float_sum_close(agg, ragg, sabs)
            else:
                assert np.array_equal(agg.astype(ragg.dtype), ragg)


@pytest.mark.parametrize("op", [0, 1, 2])
def test_reduce_by_key_run_lengths(cuda, op):
    for i, n in enumerate(SIZES):
        for mean_run in (1.0, 2.5, 100, 50000, 10 * n):
            keys = run_keys(n, mean_run, np.int32, seed=7 * i)
            vals = values_of(n, np.uint32, seed=i)
            uk, agg, r = abi_reduce_by_key(op, keys, vals, offset_elems=i % 2)
            ruk, ragg, rr = oracle.reduce_by_key(op, keys, vals)
            assert r == rr and np.array_equal(uk, ruk) and np.array_equal(agg, ragg), (n, mean_run)


def test_float_key_equality(cuda):
    # value comparison: -0 == +0 share a run (key of the run's last item), NaN never equal
    k = np.array([0.0, -0.0, np.nan, np.nan, 1.0, 1.0], dtype=np.float32)
    v = np.arange(1, 7, dtype=np.int32)
    uk, agg, r = abi_reduce_by_key(0, k, v)
    ruk, ragg, rr = oracle.reduce_by_key(0, k, v)
    assert r == rr == 4 and agg.tolist() == ragg.tolist()
    assert np.array_equal(uk.view(np.uint32), ruk.view(np.uint32))
    assert np.array_equal(abi_scan_by_key(False, 0, k, v), oracle.scan_by_key(False, 0, k, v))


def test_empty_and_in_place(cuda):
    from lc_parallel_primitive_b200 import _lib as L

    uk, agg, r = abi_reduce_by_key(0, np.zeros(0, np.int32), np.zeros(0, np.int32))
    assert r == 0
    assert L.lib().lcpp_scan_by_key(0, 0, L.I32, L.I32, None, None, None, 0, None, None, 0, None) == 0
    keys = run_keys(123457, 40, np.uint32, seed=3)
    vals = values_of(123457, np.uint32, seed=4)
    got = abi_scan_by_key(True, 0, keys, vals, in_place=True)
    assert np.array_equal(got, oracle.scan_by_key(True, 0, keys, vals))


def test_large_properties(cuda):
    # 2^28 items (the bench size): keys i // L, values 1 -> exclusive i % L,
    # inclusive i % L + 1; runs = ceil(n / L), every aggregate L (last: rest).
    import torch
    from lc_parallel_primitive_b200 import _lib as L

    lib = L.lib()
    n, Lr = 1 << 28, 777
    idx = torch.arange(n, device=cuda, dtype=torch.int64)
    keys = (idx // Lr).to(torch.int32)
    vals = torch.ones(n, dtype=torch.int32, device=cuda)
    out = torch.empty(n, dtype=torch.int32, device=cuda)
    s = torch.cuda.current_stream().cuda_stream
    tb = lib.lcpp_scan_by_key_temp_bytes(L.I32, L.I32, n)
    t = torch.empty(tb, dtype=torch.uint8, device=cuda)
    L.check(lib.lcpp_scan_by_key(0, 0, L.I32, L.I32, keys.data_ptr(), vals.data_ptr(), out.data_ptr(), n,
                                 None, t.data_ptr(), tb, s))
    torch.cuda.synchronize()
    assert torch.equal(out, (idx % Lr).to(torch.int32))
    runs = (n + Lr - 1) // Lr
    uk = torch.empty(runs, dtype=torch.int32, device=cuda)
    agg = torch.empty(runs, dtype=torch.int32, device=cuda)
    nr = torch.zeros(1, dtype=torch.int32, device=cuda)
    L.check(lib.lcpp_reduce_by_key(0, L.I32, L.I32, keys.data_ptr(), vals.data_ptr(), uk.data_ptr(),
                                   agg.data_ptr(), nr.data_ptr(), n, t.data_ptr(), tb, s))
    torch.cuda.synchronize()
    assert int(nr.item()) == runs
    assert torch.equal(uk, torch.arange(runs, device=cuda, dtype=torch.int32))
    assert torch.all(agg[:-1] == Lr) and int(agg[-1].item()) == n - (runs - 1) * Lr
    L.check(lib.lcpp_last_device_error(s))
