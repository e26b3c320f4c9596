"""Multi-GPU reduce / scan / sort on 2+ NCCL ranks (one process per GPU),
checked against the CPU oracle.  Skipped with fewer than 2 GPUs."""
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parent.parent


def test_mg_primitives_nccl(cuda):
    import torch

    ngpu = torch.cuda.device_count()
    if ngpu < 2:
        pytest.skip("needs 2 or more GPUs")
    n = min(ngpu, 4)
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run([sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
                        "--master-addr", "127.0.0.1", "--master-port", "29533",
                        str(ROOT / "tests" / "mg_gpu_worker.py")], capture_output=True, text=True, timeout=600,
                       env=env, cwd=str(ROOT))
    assert r.returncode == 0 and "MG_OK" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]
