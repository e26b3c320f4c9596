"""ctypes binding of liblcpp_b200.so (the C ABI declared in include/lcpp_b200.h).

The library is loaded from the package directory only.  There is no fallback:
if the shared object is missing or does not load, every call raises.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "liblcpp_b200.so"
DATAGEN_PATH = _PKG / "libpcg_datagen.so"

# lcpp_dtype
I32, U32, F32, I64, U64, F64, NONE = 0, 1, 2, 3, 4, 5, 15
# lcpp_op
OP_SUM, OP_MIN, OP_MAX = 0, 1, 2
# lcpp_scan_kind
SCAN_EXCLUSIVE, SCAN_INCLUSIVE = 0, 1
XF_IDENTITY, XF_SQUARE, XF_ABS, XF_NEGATE = 0, 1, 2, 3
# lcpp_status
OK = 0
ERR_INVALID_ARG = -1
ERR_TEMP_TOO_SMALL = -2
ERR_CUDA = -3
ERR_LOOKBACK_TIMEOUT = -4
ERR_NCCL = -5
ERR_UNSUPPORTED = -6
ERR_CAPACITY = -7

_vp, _u64, _sz, _i, _u32 = C.c_void_p, C.c_uint64, C.c_size_t, C.c_int, C.c_uint32

# name -> (restype, argtypes); the complete list of symbols of include/lcpp_b200.h
SIGNATURES = {
    "lcpp_status_string": (C.c_char_p, [_i]),
    "lcpp_dtype_size": (_sz, [_i]),
    "lcpp_reduce_temp_bytes": (_sz, [_i, _u64]),
    "lcpp_reduce": (_i, [_i, _i, _vp, _vp, _u64, _vp, _sz, _vp]),
    "lcpp_scan_temp_bytes": (_sz, [_i, _u64]),
    "lcpp_scan": (_i, [_i, _i, _vp, _vp, _u64, _vp, _sz, _vp]),
    "lcpp_scan_carry": (_i, [_i, _i, _vp, _vp, _u64, _vp, _vp, _sz, _vp]),
    "lcpp_scan_op": (_i, [_i, _i, _i, _vp, _vp, _u64, _vp, _vp, _sz, _vp]),
    "lcpp_scan_noalloc_max_items": (_u64, []),
    "lcpp_scan_noalloc": (_i, [_i, _i, _vp, _vp, _u64, _vp]),
    "lcpp_radix_sort_temp_bytes": (_sz, [_i, _i, _u64]),
    "lcpp_radix_sort": (_i, [_i, _i, _i, _vp, _vp, _vp, _vp, _u64, _i, _i, _vp, _sz, _vp]),
    "lcpp_radix_bucket_starts": (_i, [_i, _vp, _u64, _i, _vp, _vp]),
    "lcpp_segment_reduce_temp_bytes": (_sz, [_i, _u64, _u64]),
    "lcpp_segment_reduce": (_i, [_i, _i, _vp, _vp, _u64, _vp, _vp, _vp, _sz, _vp]),
    "lcpp_segment_reduce_fixed": (_i, [_i, _i, _vp, _vp, _u64, _u64, _vp]),
    "lcpp_arg_reduce_temp_bytes": (_sz, [_i, _u64]),
    "lcpp_arg_reduce": (_i, [_i, _i, _vp, _vp, _vp, _u64, _vp, _sz, _vp]),
    "lcpp_segment_arg_reduce": (_i, [_i, _i, _vp, _vp, _vp, _u64, _vp, _vp, _vp]),
    "lcpp_segment_arg_reduce_fixed": (_i, [_i, _i, _vp, _vp, _vp, _u64, _u64, _vp]),
    "lcpp_transform_reduce": (_i, [_i, _i, _i, _vp, _vp, _u64, _vp, _vp, _sz, _vp]),
    "lcpp_scan_by_key_temp_bytes": (_sz, [_i, _i, _u64]),
    "lcpp_scan_by_key": (_i, [_i, _i, _i, _i, _vp, _vp, _vp, _u64, _vp, _vp, _sz, _vp]),
    "lcpp_reduce_by_key_temp_bytes": (_sz, [_i, _i, _u64]),
    "lcpp_reduce_by_key": (_i, [_i, _i, _i, _vp, _vp, _vp, _vp, _vp, _u64, _vp, _sz, _vp]),
    "lcpp_mg_unique_id_bytes": (_sz, []),
    "lcpp_mg_get_unique_id": (_i, [_vp]),
    "lcpp_mg_comm_init_rank": (_i, [C.POINTER(_vp), _i, _vp, _i]),
    "lcpp_mg_comm_destroy": (_i, [_vp]),
    "lcpp_mg_comm_shape": (_i, [_vp, C.POINTER(_i), C.POINTER(_i)]),
    "lcpp_mg_reduce_temp_bytes": (_sz, [_i, _u64]),
    "lcpp_mg_reduce": (_i, [_i, _i, _vp, _vp, _u64, _vp, _sz, _vp, _vp]),
    "lcpp_mg_scan_temp_bytes": (_sz, [_i, _u64, _i]),
    "lcpp_mg_scan": (_i, [_i, _i, _vp, _vp, _u64, _vp, _sz, _vp, _vp]),
    "lcpp_mg_sort_temp_bytes": (_sz, [_i, _i, _u64, _u64, _i]),
    "lcpp_mg_sort": (_i, [_i, _i, _vp, _vp, _u64, _vp, _vp, _u64, C.POINTER(_u64), _vp, _sz, _vp, _vp]),
    "lcpp_mg_pick_splitters": (_i, [C.POINTER(_u64), C.POINTER(_u64), C.POINTER(_u64), _u64, _i,
                                    C.POINTER(_u64), C.POINTER(_u64)]),
    "lcpp_last_device_error": (_i, [_vp]),
    "lcpp_lookback_temp_bytes": (_sz, [_u64]),
    "lcpp_lookback_tiles": (_i, [_vp, _vp, _vp, _u64, _vp, _sz, _vp]),
    "lcpp_set_spin_limit": (_i, [_u32]),
    "lcpp_lookback_probe": (_i, [_vp, _u64, _vp, _vp]),
    "lcpp_profile_enable": (_i, [_i]),
    "lcpp_profile_read": (_i, [C.c_char_p, C.POINTER(_u64), C.POINTER(C.c_double)]),
    "lcpp_kernel_launch_count": (_u64, []),
    "lcpp_kernel_binary_version": (_i, []),
    "lcpp_build_info": (C.c_char_p, []),
}


class LcppError(RuntimeError):
    def __init__(self, status: int, what: str = ""):
        self.status = status
        msg = _status_string(status)
        super().__init__(f"{what}: {msg} ({status})" if what else f"{msg} ({status})")


_lib = None


def lib() -> C.CDLL:
    """The loaded liblcpp_b200.so (raises if it is not built or fails to load)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH} is not built; run `python -m lc_parallel_primitive_b200.build` "
                "(or __graft_entry__.build())")
        h = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            f = getattr(h, name)
            f.restype = res
            f.argtypes = args
        _lib = h
    return _lib


def _status_string(s: int) -> str:
    try:
        return lib().lcpp_status_string(s).decode()
    except Exception:  # library not loadable: still give a readable message
        return {0: "ok", -1: "invalid argument", -2: "temp storage too small", -3: "CUDA error",
                -4: "look-back wait timed out", -5: "NCCL error", -6: "unsupported", -7: "output capacity exceeded"}.get(s, "status")


def check(status: int, what: str = "") -> None:
    if status != OK:
        raise LcppError(status, what)


_datagen = None


def datagen() -> C.CDLL:
    global _datagen
    if _datagen is None:
        if not DATAGEN_PATH.exists():
            raise RuntimeError(f"{DATAGEN_PATH} is not built")
        h = C.CDLL(str(DATAGEN_PATH))
        h.pcg_fill.restype = _i
        h.pcg_fill.argtypes = [_i, _vp, _u64, _u64, _u64, C.c_int64, C.c_int64, _i]
        h.fill_iota_u32.restype = None
        h.fill_iota_u32.argtypes = [_vp, _u64, _u32]
        h.pcg_segments_lognormal.restype = _i
        h.pcg_segments_lognormal.argtypes = [_vp, _u64, _u64, C.c_double, C.c_double, C.c_double, _u64, _u64]
        _datagen = h
    return _datagen
