"""All-gather GEMM on 2+ GPUs: spawns torch.distributed.run with one rank per GPU.  Gathered
bytes must equal an NCCL all-gather, the gated GEMM must be bitwise equal to the dense GEMM on
the gathered operands, over several iterations (buffer rotation) and with a late sender."""

import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_all_gather_gemm_multi_gpu():
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs at least 2 GPUs")
    world = 2 if n < 4 else 4
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", NCCL_MAX_CTAS="16")
    worker = os.path.join(os.path.dirname(os.path.abspath(__file__)), "dist_worker.py")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={world}",
           "--master-addr", "127.0.0.1", "--master-port", "29611", worker]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "DIST_WORKER_OK" in r.stdout, (r.stdout[-3000:], r.stderr[-3000:])
