"""Multi-GPU C ABI (lcpp_mg_*) on NCCL communicators: one rank in-process
(runs on a 1-GPU box) and 2+ ranks under torchrun (skipped with fewer GPUs),
checked against the CPU oracle."""
import ctypes as C
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

import oracle
from tests.helpers import empty_dev, stream, to_dev, to_host

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent


@pytest.fixture(scope="module")
def comm1(cuda):
    """A 1-rank NCCL communicator made through the library's helpers."""
    from lc_parallel_primitive_b200 import _lib as L

    lib = L.lib()
    uid = C.create_string_buffer(int(lib.lcpp_mg_unique_id_bytes()))
    L.check(lib.lcpp_mg_get_unique_id(uid))
    h = C.c_void_p()
    L.check(lib.lcpp_mg_comm_init_rank(C.byref(h), 1, uid, 0))
    r, n = C.c_int(-1), C.c_int(-1)
    L.check(lib.lcpp_mg_comm_shape(h, C.byref(r), C.byref(n)))
    assert (r.value, n.value) == (0, 1)
    yield h
    L.check(lib.lcpp_mg_comm_destroy(h))


def _temp(nb):
    import torch

    return torch.empty(max(int(nb), 1), dtype=torch.uint8, device="cuda")


@pytest.mark.parametrize("n", [0, 1, 4097, 1 << 20])
def test_mg_single_rank_matches_oracle(comm1, n):
    from lc_parallel_primitive_b200 import _lib as L
    from lc_parallel_primitive_b200 import datagen as G

    lib = L.lib()
    s = stream()
    keys = G.u64(n, seed=11)
    vals = np.arange(n, dtype=np.uint32)
    dk, dv = to_dev(keys), to_dev(vals)
    ok_, ov = empty_dev(max(n, 1), np.uint64), empty_dev(max(n, 1), np.uint32)
    tb = lib.lcpp_mg_sort_temp_bytes(L.U64, L.U32, n, n, 1)
    t = _temp(tb)
    n_out = C.c_uint64(99)
    L.check(lib.lcpp_mg_sort(L.U64, L.U32, dk.data_ptr(), dv.data_ptr(), n, ok_.data_ptr(), ov.data_ptr(), n,
                             C.byref(n_out), t.data_ptr(), tb, comm1, s))
    x = G.u32(n, seed=12)
    dx = to_dev(x)
    dy = empty_dev(max(n, 1), np.uint32)
    tb2 = lib.lcpp_mg_scan_temp_bytes(L.U32, n, 1)
    t2 = _temp(tb2)
    L.check(lib.lcpp_mg_scan(L.SCAN_EXCLUSIVE, L.U32, dx.data_ptr(), dy.data_ptr(), n, t2.data_ptr(), tb2, comm1, s))
    red = empty_dev(1, np.uint32)
    tb3 = lib.lcpp_mg_reduce_temp_bytes(L.U32, n)
    t3 = _temp(tb3)
    L.check(lib.lcpp_mg_reduce(L.OP_MAX, L.U32, dx.data_ptr(), red.data_ptr(), n, t3.data_ptr(), tb3, comm1, s))
    import torch

    torch.cuda.synchronize()
    L.check(lib.lcpp_last_device_error(s))
    assert n_out.value == n
    wk, wv = oracle.radix_sort(keys, vals)
    assert np.array_equal(to_host(ok_)[:n], wk) and np.array_equal(to_host(ov)[:n], wv)
    assert np.array_equal(to_host(dy)[:n], oracle.scan(False, x))
    assert int(to_host(red)[0]) == (int(x.max()) if n else 0)


def test_mg_rejects_bad_arguments(comm1):
    from lc_parallel_primitive_b200 import _lib as L

    lib = L.lib()
    n_out = C.c_uint64(0)
    # capacity below n_local, and a temp buffer that is too small
    assert lib.lcpp_mg_sort(L.U32, L.NONE, 1, None, 10, 1, None, 5, C.byref(n_out), 1, 1 << 20, comm1,
                            None) == L.ERR_INVALID_ARG
    assert lib.lcpp_mg_sort(L.U32, L.NONE, 1, None, 10, 1, None, 10, C.byref(n_out), 1, 16, comm1,
                            None) == L.ERR_TEMP_TOO_SMALL
    assert lib.lcpp_mg_reduce(0, L.U32, 1, 1, 10, 1, 16, None, None) in (L.ERR_NCCL, L.ERR_TEMP_TOO_SMALL)


@pytest.mark.parametrize("exchange", ["ipc", "nccl"])
def test_mg_primitives_nccl(cuda, exchange):
    """2-4 ranks; the sort's exchange by CUDA IPC pulls (default) and by NCCL
    send/recv (LCPP_MG_EXCHANGE=nccl)."""
    import torch

    ngpu = torch.cuda.device_count()
    if ngpu < 2:
        pytest.skip("needs 2 or more GPUs")
    n = min(ngpu, 4)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    if exchange == "nccl":
        env["LCPP_MG_EXCHANGE"] = "nccl"
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
                        "--master-addr", "127.0.0.1", "--master-port", str(29533 + (exchange == "nccl")),
                        str(ROOT / "tests" / "mg_gpu_worker.py")], capture_output=True, text=True, timeout=600,
                       env=env, cwd=str(ROOT))
    assert r.returncode == 0 and "MG_OK" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]
    assert f"nranks={n}" in r.stdout
