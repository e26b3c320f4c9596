"""Shared helpers for the parity tests: numpy <-> CUDA tensors, direct C-ABI
calls, golden-case regeneration and tolerance checks."""
from __future__ import annotations

import subprocess
import tempfile
from pathlib import Path

import numpy as np

from lc_parallel_primitive_b200 import _lib as L

ROOT = Path(__file__).resolve().parent.parent
GOLDEN = ROOT / "tests" / "golden"


def to_dev(a: np.ndarray, offset_elems: int = 0):
    """Copy a numpy array to a CUDA tensor; with offset_elems > 0 the result is
    a view starting offset_elems elements into a larger buffer (unaligned base)."""
    import torch

    t = torch.from_numpy(np.ascontiguousarray(a))
    if offset_elems:
        big = torch.empty(a.size + offset_elems, dtype=t.dtype, device="cuda")
        big[offset_elems:].copy_(t)
        return big[offset_elems:]
    return t.to("cuda")


def to_host(t) -> np.ndarray:
    return t.cpu().numpy()


def empty_dev(n, np_dtype, offset_elems: int = 0):
    import torch

    dt = {np.dtype(np.int32): torch.int32, np.dtype(np.uint32): torch.uint32,
          np.dtype(np.float32): torch.float32, np.dtype(np.int64): torch.int64,
          np.dtype(np.uint64): torch.uint64, np.dtype(np.float64): torch.float64}[np.dtype(np_dtype)]
    big = torch.empty(n + offset_elems, dtype=dt, device="cuda")
    return big[offset_elems:] if offset_elems else big


def temp(nbytes):
    import torch

    return torch.empty(max(nbytes, 1), dtype=torch.uint8, device="cuda")


def stream():
    import torch

    return torch.cuda.current_stream().cuda_stream


NP2LCPP = {np.dtype(np.int32): L.I32, np.dtype(np.uint32): L.U32, np.dtype(np.float32): L.F32,
           np.dtype(np.int64): L.I64, np.dtype(np.uint64): L.U64, np.dtype(np.float64): L.F64}


def abi_reduce(op, x_np, offset_elems=0):
    import torch

    lib = L.lib()
    d = to_dev(x_np, offset_elems)
    out = empty_dev(1, x_np.dtype)
    dt = NP2LCPP[x_np.dtype]
    tb = lib.lcpp_reduce_temp_bytes(dt, x_np.size)
    t = temp(tb)
    L.check(lib.lcpp_reduce(op, dt, d.data_ptr(), out.data_ptr(), x_np.size, t.data_ptr(), tb, stream()))
    torch.cuda.synchronize()
    L.check(lib.lcpp_last_device_error(stream()))
    return to_host(out)[0]


def abi_scan(inclusive, x_np, offset_elems=0, in_place=False):
    import torch

    lib = L.lib()
    d = to_dev(x_np, offset_elems)
    out = d if in_place else empty_dev(x_np.size, x_np.dtype, offset_elems)
    dt = NP2LCPP[x_np.dtype]
    tb = lib.lcpp_scan_temp_bytes(dt, x_np.size)
    t = temp(tb)
    L.check(lib.lcpp_scan(int(inclusive), dt, d.data_ptr(), out.data_ptr(), x_np.size, t.data_ptr(), tb,
                          stream()))
    torch.cuda.synchronize()
    L.check(lib.lcpp_last_device_error(stream()))
    return to_host(out)


def abi_sort(keys_np, values_np=None, descending=False, begin_bit=0, end_bit=0, offset_elems=0):
    import torch

    lib = L.lib()
    kd = NP2LCPP[keys_np.dtype]
    vd = L.NONE if values_np is None else NP2LCPP[values_np.dtype]
    ki = to_dev(keys_np, offset_elems)
    ko = empty_dev(keys_np.size, keys_np.dtype, offset_elems)
    vi = vo = None
    if values_np is not None:
        vi = to_dev(values_np, offset_elems)
        vo = empty_dev(values_np.size, values_np.dtype, offset_elems)
    tb = lib.lcpp_radix_sort_temp_bytes(kd, vd, keys_np.size)
    t = temp(tb)
    L.check(lib.lcpp_radix_sort(kd, vd, int(descending), ki.data_ptr(), ko.data_ptr(),
                                None if vi is None else vi.data_ptr(), None if vo is None else vo.data_ptr(),
                                keys_np.size, begin_bit, end_bit, t.data_ptr(), tb, stream()))
    torch.cuda.synchronize()
    L.check(lib.lcpp_last_device_error(stream()))
    if values_np is None:
        return to_host(ko)
    return to_host(ko), to_host(vo)


def abi_segment_reduce(op, x_np, begin_np, end_np, with_temp=True):
    import torch

    lib = L.lib()
    dt = NP2LCPP[x_np.dtype]
    d = to_dev(x_np)
    b = to_dev(begin_np.astype(np.uint32))
    e = to_dev(end_np.astype(np.uint32))
    S = begin_np.size
    out = empty_dev(S, x_np.dtype)
    tb = lib.lcpp_segment_reduce_temp_bytes(dt, x_np.size, S) if with_temp else 0
    t = temp(tb) if with_temp else None
    L.check(lib.lcpp_segment_reduce(op, dt, d.data_ptr(), out.data_ptr(), S, b.data_ptr(), e.data_ptr(),
                                    None if t is None else t.data_ptr(), tb, stream()))
    torch.cuda.synchronize()
    L.check(lib.lcpp_last_device_error(stream()))
    return to_host(out)


def abi_segment_reduce_fixed(op, x_np, num_segments, seg_size):
    import torch

    lib = L.lib()
    dt = NP2LCPP[x_np.dtype]
    d = to_dev(x_np)
    out = empty_dev(num_segments, x_np.dtype)
    L.check(lib.lcpp_segment_reduce_fixed(op, dt, d.data_ptr(), out.data_ptr(), num_segments, seg_size,
                                          stream()))
    torch.cuda.synchronize()
    return to_host(out)


def abi_scan_by_key(inclusive, op, keys_np, values_np, init=None, offset_elems=0, in_place=False, temp_buf=None):
    import torch

    lib = L.lib()
    kdt, vdt = NP2LCPP[keys_np.dtype], NP2LCPP[values_np.dtype]
    n = values_np.size
    k = to_dev(keys_np, offset_elems)
    v = to_dev(values_np, offset_elems)
    out = v if in_place else empty_dev(n, values_np.dtype, offset_elems)
    tb = lib.lcpp_scan_by_key_temp_bytes(kdt, vdt, n)
    t = temp(tb) if temp_buf is None else temp_buf  # a caller's buffer may hold another call's state
    iv = None if init is None else np.array([init], dtype=values_np.dtype)
    L.check(lib.lcpp_scan_by_key(L.SCAN_INCLUSIVE if inclusive else L.SCAN_EXCLUSIVE, op, kdt, vdt,
                                 k.data_ptr(), v.data_ptr(), out.data_ptr(), n,
                                 None if iv is None else iv.ctypes.data, t.data_ptr(), tb, stream()))
    torch.cuda.synchronize()
    L.check(lib.lcpp_last_device_error(stream()))
    return to_host(out)


def abi_reduce_by_key(op, keys_np, values_np, offset_elems=0):
    """(unique_keys, aggregates, num_runs) from the device."""
    import torch

    lib = L.lib()
    kdt, vdt = NP2LCPP[keys_np.dtype], NP2LCPP[values_np.dtype]
    n = values_np.size
    k = to_dev(keys_np, offset_elems)
    v = to_dev(values_np, offset_elems)
    uk = empty_dev(max(n, 1), keys_np.dtype)
    agg = empty_dev(max(n, 1), values_np.dtype)
    nr = torch.full((1,), 0xDEAD, dtype=torch.int32, device="cuda")
    tb = lib.lcpp_reduce_by_key_temp_bytes(kdt, vdt, n)
    t = temp(tb)
    L.check(lib.lcpp_reduce_by_key(op, kdt, vdt, k.data_ptr(), v.data_ptr(), uk.data_ptr(), agg.data_ptr(),
                                   nr.data_ptr(), n, t.data_ptr(), tb, stream()))
    torch.cuda.synchronize()
    L.check(lib.lcpp_last_device_error(stream()))
    r = int(nr.cpu().numpy().view(np.uint32)[0])
    return to_host(uk)[:r], to_host(agg)[:r], r


# ---- reference-test regeneration (tests/golden/refgen.cpp) -----------------
def refgen(case: str, n: int = 0) -> dict:
    from oracle.build import build_refgen

    exe = build_refgen()
    with tempfile.TemporaryDirectory() as d:
        cmd = [str(exe), case, d] + ([str(n)] if n else [])
        subprocess.run(cmd, check=True)
        out = {}
        for p in Path(d).glob("*.bin"):
            name, dt, _ = p.name.rsplit(".", 2)
            out[name] = np.fromfile(p, dtype={"i32": np.int32, "u32": np.uint32, "f32": np.float32}[dt])
        return out


# ---- tolerances --------------------------------------------------------------
def assert_float_sum_close(y, ref_fp64, abs_scale, rel=1e-5):
    """|y - ref| <= rel * max(|ref|, abs_scale * 2^-6): fp32 results within
    1e-5 relative of an fp64 oracle, with the relative scale floored at
    1/64 of the running sum of |x| (abs_scale) where prefixes cross zero.
    The floor is the conditioning term of floating-point summation: any fp32
    summation order (sequential included) carries an error of order
    u * sum|x| (u = 2^-24), so the floor must exceed u / rel ~ 2^-7.4; 2^-6
    is the smallest power of two above that.  Measured on B200: the N(0,1)
    InclusiveSum / ExclusiveSum at 2^24-2^28 items stay at 0.08 of this
    bound, and a 2^-10 floor is exceeded (ratio 1.2 at item 109 of the
    float scan tests' input)."""
    y = np.asarray(y, dtype=np.float64)
    ref = np.asarray(ref_fp64, dtype=np.float64)
    scale = np.maximum(np.abs(ref), np.asarray(abs_scale, dtype=np.float64) * 2.0 ** -6)
    err = np.abs(y - ref)
    bad = err > rel * scale + 1e-30
    if bad.any():
        i = int(np.argmax(bad))
        raise AssertionError(f"{int(bad.sum())} elements out of tolerance; first at {i}: "
                             f"got {y[i]!r} want {ref[i]!r} (scale {scale[i]!r})")
