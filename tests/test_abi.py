"""C ABI checks that need no GPU: the library loads, exports every function
declared in include/*.h, and validates arguments before touching the device."""
import ctypes
import re
from pathlib import Path

import pytest

from lc_parallel_primitive_b200 import _lib as L

ROOT = Path(__file__).resolve().parent.parent


def declared_functions(header: Path):
    text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
    text = re.sub(r"//[^\n]*", "", text)
    return sorted(set(re.findall(r"\b(lcpp_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = L.lib()
    names = declared_functions(ROOT / "include" / "lcpp_b200.h")
    assert len(names) >= 19
    for name in names:
        assert hasattr(lib, name), name
    assert set(names) == set(L.SIGNATURES), set(names) ^ set(L.SIGNATURES)


@pytest.mark.gpu
def test_library_is_sm100a(cuda):
    """The loaded kernels are sm_100a code (cudaFuncGetAttributes binaryVersion)."""
    assert L.lib().lcpp_kernel_binary_version() == 100


def test_temp_sizes():
    lib = L.lib()
    assert lib.lcpp_reduce_temp_bytes(L.I32, 1 << 24) > 0
    assert lib.lcpp_reduce_temp_bytes(L.NONE, 10) == 0
    assert lib.lcpp_scan_temp_bytes(L.U32, 1 << 28) >= 8 * (1 << 28) // 8192
    assert lib.lcpp_scan_temp_bytes(L.U64, 1 << 28) > lib.lcpp_scan_temp_bytes(L.U32, 1 << 28)  # 8-byte descriptors
    assert lib.lcpp_scan_temp_bytes(L.NONE, 10) == 0
    n = 1 << 28
    pairs = lib.lcpp_radix_sort_temp_bytes(L.U32, L.U32, n)
    keys = lib.lcpp_radix_sort_temp_bytes(L.U32, L.NONE, n)
    assert pairs >= 8 * n and keys >= 4 * n and pairs > keys
    assert lib.lcpp_radix_sort_temp_bytes(L.NONE, L.NONE, 10) == 0
    assert lib.lcpp_segment_reduce_temp_bytes(L.F32, 1 << 27, 1 << 20) >= 4 << 20
    assert lib.lcpp_dtype_size(L.F64) == 8 and lib.lcpp_dtype_size(L.NONE) == 0


def test_argument_validation_without_device():
    lib = L.lib()
    bad = ctypes.c_void_p(16)
    assert lib.lcpp_reduce(7, L.I32, bad, bad, 10, bad, 1 << 20, None) == L.ERR_INVALID_ARG
    assert lib.lcpp_reduce(0, 99, bad, bad, 10, bad, 1 << 20, None) == L.ERR_INVALID_ARG
    assert lib.lcpp_reduce(0, L.I32, bad, bad, 10, bad, 16, None) == L.ERR_TEMP_TOO_SMALL
    assert lib.lcpp_scan(5, L.U32, bad, bad, 10, bad, 1 << 20, None) == L.ERR_INVALID_ARG
    assert lib.lcpp_scan(0, L.NONE, bad, bad, 10, bad, 1 << 20, None) == L.ERR_INVALID_ARG
    assert lib.lcpp_scan(0, L.U32, bad, bad, 0, None, 0, None) == L.OK  # n = 0: nothing to do
    assert lib.lcpp_scan(0, L.U32, bad, bad, 1 << 20, bad, 8, None) == L.ERR_TEMP_TOO_SMALL
    assert lib.lcpp_radix_sort(L.NONE, L.NONE, 0, bad, bad, None, None, 10, 0, 0, bad, 1 << 30, None) == L.ERR_INVALID_ARG
    assert lib.lcpp_radix_sort(L.U32, L.NONE, 0, bad, bad, None, None, 1 << 32, 0, 0, bad, 1 << 40, None) == L.ERR_INVALID_ARG
    assert lib.lcpp_radix_sort(L.U32, L.NONE, 0, bad, bad, None, None, 10, 0, 33, bad, 1 << 20, None) == L.ERR_INVALID_ARG
    assert lib.lcpp_radix_sort(L.U32, L.NONE, 0, bad, bad, None, None, 10, 8, 8, bad, 1 << 20, None) == L.ERR_INVALID_ARG
    assert lib.lcpp_radix_sort(L.U32, L.U32, 0, bad, bad, None, None, 10, 0, 0, bad, 1 << 20, None) == L.ERR_INVALID_ARG
    assert lib.lcpp_radix_sort(L.U32, L.NONE, 0, bad, bad, None, None, 1 << 20, 0, 0, bad, 64, None) == L.ERR_TEMP_TOO_SMALL
    assert lib.lcpp_segment_reduce(3, L.F32, bad, bad, 10, bad, bad, bad, 1 << 20, None) == L.ERR_INVALID_ARG
    assert lib.lcpp_segment_reduce(0, L.F32, bad, bad, 0, None, None, None, 0, None) == L.OK
    assert lib.lcpp_lookback_tiles(None, None, None, 5, bad, 1 << 20, None) == L.ERR_INVALID_ARG


def test_status_strings():
    lib = L.lib()
    assert lib.lcpp_status_string(L.ERR_LOOKBACK_TIMEOUT) == b"look-back wait timed out"
    err = L.LcppError(L.ERR_TEMP_TOO_SMALL, "DeviceScan")
    assert "temp storage too small" in str(err) and err.status == L.ERR_TEMP_TOO_SMALL
