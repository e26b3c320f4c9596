"""The scan's decoupled look-back on its own (reference test
tests/decoupled_look_back.cpp:57-180) and its bounded wait."""
import numpy as np
import pytest

from lc_parallel_primitive_b200 import _lib as L
from tests.helpers import abi_reduce, stream, temp

pytestmark = pytest.mark.gpu


def test_reference_lookback_tiles_of_one(cuda):
    # 102400 tiles, each aggregate 1: exclusive = i, inclusive = i + 1.
    import torch

    lib = L.lib()
    T = 102400
    agg = torch.ones(T, dtype=torch.int32, device=cuda)
    ex = torch.empty(T, dtype=torch.int32, device=cuda)
    inc = torch.empty(T, dtype=torch.int32, device=cuda)
    tb = lib.lcpp_lookback_temp_bytes(T)
    t = temp(tb)
    L.check(lib.lcpp_lookback_tiles(agg.data_ptr(), ex.data_ptr(), inc.data_ptr(), T, t.data_ptr(), tb, stream()))
    torch.cuda.synchronize()
    L.check(lib.lcpp_last_device_error(stream()))
    assert np.array_equal(ex.cpu().numpy(), np.arange(T))
    assert np.array_equal(inc.cpu().numpy(), np.arange(T) + 1)


def test_lookback_over_published_descriptors(cuda):
    import torch

    lib = L.lib()
    # tiles 0..9: tile 0 inclusive 5, tiles 1..8 partial 1..8 -> prefix of tile 9 = 5 + 36
    desc = np.zeros(10, dtype=np.uint64)
    desc[0] = (2 << 32) | 5
    for i in range(1, 9):
        desc[i] = (1 << 32) | i
    d = torch.from_numpy(desc.view(np.int64)).to(cuda)
    out = torch.zeros(1, dtype=torch.int32, device=cuda)
    L.check(lib.lcpp_lookback_probe(d.data_ptr(), 9, out.data_ptr(), stream()))
    torch.cuda.synchronize()
    assert lib.lcpp_last_device_error(stream()) == L.OK
    assert int(out.cpu()[0]) == 5 + 36


def test_unpublished_predecessor_times_out(cuda):
    # A predecessor that never publishes: the wait runs out after the cap,
    # the kernel returns, the host reads LOOKBACK_TIMEOUT, the context stays
    # usable.  Nothing traps or hangs.
    import torch

    lib = L.lib()
    desc = torch.zeros(64, dtype=torch.int64, device=cuda)  # nothing published
    out = torch.zeros(1, dtype=torch.int32, device=cuda)
    L.check(lib.lcpp_set_spin_limit(1000))
    try:
        L.check(lib.lcpp_lookback_probe(desc.data_ptr(), 40, out.data_ptr(), stream()))
        torch.cuda.synchronize()
        assert lib.lcpp_last_device_error(stream()) == L.ERR_LOOKBACK_TIMEOUT
        assert lib.lcpp_last_device_error(stream()) == L.OK  # cleared by the read
    finally:
        L.check(lib.lcpp_set_spin_limit(0))
    x = np.arange(1000, dtype=np.int32)
    assert abi_reduce(0, x) == x.sum()
