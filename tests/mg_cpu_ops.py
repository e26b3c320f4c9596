"""CPU stand-in for GpuOps, used only by the gloo tests of the multi-GPU host
logic (the library itself has no CPU path)."""
import numpy as np
import torch

import oracle

_NP = {torch.int32: np.int32, torch.uint32: np.uint32, torch.float32: np.float32,
       torch.int64: np.int64, torch.uint64: np.uint64, torch.float64: np.float64}


def _np(t):
    return t.numpy()


class CpuOps:
    def reduce(self, op, x):
        r = oracle.reduce(op, _np(x))
        return torch.tensor([r], dtype=x.dtype) if x.dtype.is_floating_point else \
            torch.from_numpy(np.array([r], dtype=_NP[x.dtype]))

    def scan(self, inclusive, x, out, carry):
        y = oracle.scan(inclusive, _np(x))
        if x.dtype == torch.float32:
            y = y.astype(np.float32)
        if carry is not None:
            c = _np(carry)[0]
            y = (y + c).astype(y.dtype) if x.dtype != torch.float32 else (y + np.float32(c)).astype(np.float32)
        out.copy_(torch.from_numpy(np.ascontiguousarray(y)))

    def bucket_starts(self, keys, bit_start):
        k = _np(keys).astype(np.uint64)
        if keys.dtype in (torch.int32, torch.int64):
            k = (_np(keys).astype(np.int64) + (1 << (keys.element_size() * 8 - 1))).astype(np.uint64)
        d = (k >> np.uint64(bit_start)) & np.uint64(0xFF)
        return torch.from_numpy(np.searchsorted(d, np.arange(257, dtype=np.uint64), side="left").astype(np.int64))

    def sort_pairs(self, keys, vals, begin_bit=0, end_bit=0):
        k, v = oracle.radix_sort(_np(keys), _np(vals), begin_bit=begin_bit, end_bit=end_bit)
        return torch.from_numpy(k), torch.from_numpy(v)
