"""Seeded input generator: determinism, thread independence, distributions."""
import numpy as np

from lc_parallel_primitive_b200 import datagen as G
from lc_parallel_primitive_b200._lib import datagen


def test_pcg32_reference_vector():
    # pcg32_srandom(42, 54): first outputs of O'Neill's pcg32 demo.
    x = G.u32(6, seed=42, stream=54)
    assert x.tolist() == [0xA15C02B7, 0x7B47F409, 0xBA1D3330, 0x83D2F293, 0xBFA4784B, 0xCBED606E]


def test_thread_count_does_not_change_output():
    a = np.empty(5_000_003, dtype=np.uint32)
    b = np.empty_like(a)
    datagen().pcg_fill(2, a.ctypes.data, a.size, 7, 3, 16, 0, 1)
    datagen().pcg_fill(2, b.ctypes.data, b.size, 7, 3, 16, 0, 8)
    assert np.array_equal(a, b) and a.max() == 15


def test_distributions():
    x = G.i32_range(1 << 20, -1000, 1000, seed=1)
    assert x.min() == -1000 and x.max() == 1000 and abs(x.mean()) < 5
    f = G.f32_normal(1 << 20, seed=2)
    assert abs(f.mean()) < 0.01 and abs(f.std() - 1) < 0.01
    u = G.f32_unit(1 << 20, seed=3)
    assert u.min() >= 0 and u.max() < 1
    k = G.u32_masked(1 << 16, 0xFF, seed=4)
    assert k.max() <= 255


def test_lognormal_segments_cover_exactly():
    N, S = 1 << 22, 1 << 15
    off = G.lognormal_offsets(S, N, seed=1)
    lens = np.diff(off.astype(np.int64))
    assert off[0] == 0 and off[-1] == N and (lens >= 0).all()
    assert 0.01 < (lens == 0).mean() < 0.04  # ~2 % empty (plus rounding)
