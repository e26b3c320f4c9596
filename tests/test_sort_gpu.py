"""DeviceRadixSort parity on the GPU against the CPU oracle and the reference
tests' known answers (tests/device_radix_sort_one_sweep.cpp)."""
import numpy as np
import pytest

import oracle
from lc_parallel_primitive_b200 import datagen as G
from tests.helpers import abi_sort, refgen, to_host

pytestmark = pytest.mark.gpu


def test_reference_float_keys_asc_desc(cuda):
    # device_radix_sort_one_sweep.cpp:61-118 (DeviceRadixSort<128,32,4>):
    # float keys U(0,1) from mt19937(114521), n = 2^5 .. 2^24, std::sort.
    for loop in range(5, 25):
        n = 1 << loop
        g = refgen("sort_float_keys", n)
        assert np.array_equal(abi_sort(g["asc_in"]), g["asc_expected"]), n
        assert np.array_equal(abi_sort(g["desc_in"], descending=True), g["desc_expected"]), n


def test_reference_uint_reversed_iota(cuda):
    # device_radix_sort_one_sweep.cpp:120-151: keys n-1..0, n = 2^0 .. 2^23.
    import torch
    from lc_parallel_primitive_b200 import CommandList, DeviceRadixSort, Stream, synchronize, temp_buffer

    sorter = DeviceRadixSort()
    stream = Stream()
    sorter.create(None, stream)
    for loop in range(24):
        n = 1 << loop
        keys = np.arange(n - 1, -1, -1, dtype=np.uint32)
        kin = torch.from_numpy(keys).to(cuda)
        kout = torch.empty_like(kin)
        temp = temp_buffer(DeviceRadixSort.GetSortKeysTempStorageBytes(n, torch.uint32))
        cmdlist = CommandList()
        sorter.SortKeys(cmdlist, temp, kin, kout, n)
        stream << cmdlist.commit() << synchronize()
        assert np.array_equal(to_host(kout), np.arange(n, dtype=np.uint32)), n


def test_reference_pairs_uint_float(cuda):
    # device_radix_sort_one_sweep.cpp:153-279: n = 524288 shuffled-iota keys,
    # float values; ascending and descending; values compared exactly.
    g = refgen("sort_pairs_uint_float")
    k, v = abi_sort(g["keys"], g["values"])
    assert np.array_equal(k, g["keys_expected"]) and np.array_equal(v, g["values_expected"])
    k, v = abi_sort(g["desc_keys"], g["desc_values"], descending=True)
    assert np.array_equal(k, g["desc_keys_expected"]) and np.array_equal(v, g["desc_values_expected"])


SIZES = [1, 2, 31, 1000, 8191, 8192, 8193, 100003, (1 << 20) + 7]


@pytest.mark.parametrize("kdt", [np.uint32, np.int32, np.float32, np.uint64, np.int64, np.float64])
@pytest.mark.parametrize("descending", [False, True])
def test_pairs_bit_exact_vs_oracle(cuda, kdt, descending):
    for i, n in enumerate(SIZES):
        if np.dtype(kdt).itemsize == 4:
            raw = G.u32(n, seed=300 + i)
        else:
            raw = G.u64(n, seed=300 + i)
        if np.dtype(kdt).kind == "f":
            keys = (G.f32_normal(n, seed=300 + i) * 100).astype(kdt)
            keys[::7] = 0.0
            keys[3::11] = -0.0  # -0.0 and +0.0 are equal keys: order kept (stable)
        else:
            keys = raw.view(kdt)
        vals = np.arange(n, dtype=np.uint32)
        got_k, got_v = abi_sort(keys, vals, descending=descending, offset_elems=i % 2)
        want_k, want_v = oracle.radix_sort(keys, vals, descending=descending)
        assert np.array_equal(got_k.view(np.uint8), want_k.view(np.uint8)), (n, kdt)
        assert np.array_equal(got_v, want_v), (n, kdt)


@pytest.mark.parametrize("vdt", [np.uint64, np.float32])
def test_value_types(cuda, vdt):
    n = 250001
    keys = G.u32(n, seed=9)
    vals = G.u64(n, seed=10).view(np.uint64) if vdt == np.uint64 else G.f32_unit(n, seed=10)
    got_k, got_v = abi_sort(keys, vals)
    want_k, want_v = oracle.radix_sort(keys, vals)
    assert np.array_equal(got_k, want_k) and np.array_equal(got_v, want_v)


def test_keys_only_vs_oracle(cuda):
    for kdt in (np.uint32, np.uint64):
        keys = (G.u32 if kdt == np.uint32 else G.u64)(333333, seed=11)
        assert np.array_equal(abi_sort(keys), oracle.radix_sort(keys))


def test_bit_range(cuda):
    keys = G.u32(200000, seed=12)
    vals = np.arange(keys.size, dtype=np.uint32)
    for bb, eb in ((0, 8), (4, 20), (8, 32), (0, 13)):
        got = abi_sort(keys, vals, begin_bit=bb, end_bit=eb)
        want = oracle.radix_sort(keys, vals, begin_bit=bb, end_bit=eb)
        assert np.array_equal(got[0], want[0]) and np.array_equal(got[1], want[1]), (bb, eb)


def test_skewed_stability(cuda):
    # BASELINE config 3 skewed variant at reduced n: 8 bits of entropy.
    n = (1 << 22) + 11
    keys = G.u32_masked(n, 0xFF, seed=13)
    vals = np.arange(n, dtype=np.uint32)
    k, v = abi_sort(keys, vals)
    ok, ov = oracle.radix_sort(keys, vals)
    assert np.array_equal(k, ok) and np.array_equal(v, ov)


def _check_sorted_pairs(keys_in, k, v):
    """Size-independent properties for values = iota: keys ascending, the
    permutation given by the values reproduces the keys, equal keys keep
    ascending values (stability), and v is a permutation."""
    assert np.all(k[1:] >= k[:-1])
    assert np.array_equal(keys_in[v], k)
    eq = k[1:] == k[:-1]
    assert np.all(v[1:][eq] > v[:-1][eq])
    seen = np.zeros(k.size, dtype=np.bool_)
    seen[v] = True
    assert seen.all()


def test_config3_pairs_full_size(cuda):
    # SortPairs of 2^28 uint32 uniform keys, values iota.
    n = 1 << 28
    keys = G.u32(n, seed=1, stream=7)
    vals = G.iota_u32(n)
    k, v = abi_sort(keys, vals)
    _check_sorted_pairs(keys, k, v)


def test_config3_skewed_full_size(cuda):
    n = 1 << 28
    keys = G.u32_masked(n, 0xFF, seed=1, stream=8)
    vals = G.iota_u32(n)
    k, v = abi_sort(keys, vals)
    _check_sorted_pairs(keys, k, v)


def test_config3_keys_full_size_vs_oracle(cuda):
    n = 1 << 28
    keys = G.u32(n, seed=2, stream=7)
    got = abi_sort(keys)
    want = oracle.radix_sort(keys, threads=8)
    assert np.array_equal(got, want)


def test_bucket_starts(cuda):
    # run boundaries of keys partitioned by their top byte (multi-GPU sort helper)
    import torch
    from lc_parallel_primitive_b200 import _lib as L
    from tests.helpers import stream

    for kdt, bits in ((np.uint32, 32), (np.int32, 32), (np.uint64, 64)):
        n = 300001
        raw = G.u32(n, seed=21) if bits == 32 else G.u64(n, seed=21)
        keys = raw.view(kdt)
        part = abi_sort(keys, begin_bit=bits - 8, end_bit=bits)
        d = torch.from_numpy(part.view(np.int32 if bits == 32 else np.int64)).to(cuda)
        out = torch.empty(257, dtype=torch.int64, device=cuda)
        dt = {np.uint32: L.U32, np.int32: L.I32, np.uint64: L.U64}[kdt]
        L.check(L.lib().lcpp_radix_bucket_starts(dt, d.data_ptr(), n, bits - 8, out.data_ptr(), stream()))
        got = out.cpu().numpy()
        u = part.view(np.uint32 if bits == 32 else np.uint64).astype(np.uint64)
        if kdt == np.int32:
            u = u ^ np.uint64(1 << 31)
        digit = (u >> np.uint64(bits - 8)) & np.uint64(0xFF)
        want = np.searchsorted(digit, np.arange(257, dtype=np.uint64), side="left")
        assert np.array_equal(got, want), kdt


def test_keys_beyond_2p30_use_wide_lookback(cuda):
    # n >= 2^30 switches the look-back words to 64 bits; check on the device:
    # ascending order and an order-independent checksum of the multiset.
    import torch
    from lc_parallel_primitive_b200 import _lib as L
    from tests.helpers import stream, temp

    n = (1 << 30) + 12345
    lib = L.lib()
    keys = torch.randint(-(1 << 31), (1 << 31) - 1, (n,), dtype=torch.int32, device=cuda,
                         generator=torch.Generator(device=cuda).manual_seed(3))
    out = torch.empty_like(keys)
    tb = lib.lcpp_radix_sort_temp_bytes(L.U32, L.NONE, n)
    t = temp(tb)
    L.check(lib.lcpp_radix_sort(L.U32, L.NONE, 0, keys.data_ptr(), out.data_ptr(), None, None, n, 0, 0,
                                t.data_ptr(), tb, stream()))
    torch.cuda.synchronize()
    L.check(lib.lcpp_last_device_error(stream()))
    del t
    o = out.to(torch.int64) & 0xFFFFFFFF
    assert bool((o[1:] >= o[:-1]).all())
    ki = keys.to(torch.int64) & 0xFFFFFFFF
    assert int(o.sum()) == int(ki.sum())
    assert int((o * o % 1000003).sum()) == int((ki * ki % 1000003).sum())
