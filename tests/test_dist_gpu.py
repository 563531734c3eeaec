"""GPU, 2 ranks over NCCL: the N-sharded GEMM + all-gather + interleave on
real devices (skipped with fewer than two GPUs)."""
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def test_sharded_gemm_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", f"--master-port={port}",
           str(ROOT / "tests" / "_dist_gpu_worker.py")]
    res = subprocess.run(cmd, capture_output=True, text=True, cwd=ROOT, env=dict(os.environ))
    assert res.returncode == 0 and "DIST_GPU_OK" in res.stdout, res.stdout[-2000:] + res.stderr[-3000:]
