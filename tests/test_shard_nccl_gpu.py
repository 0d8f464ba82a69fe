"""Multi-GPU shard driver on real GPUs: 2 ranks over NCCL (NVLink on a B200 box).

tests/shard_nccl_worker.py runs under torchrun, one rank per GPU; each rank
checks the gathered C against the CPU oracle.  Skipped with fewer than two
GPUs (the host-side logic is covered on CPU by tests/test_shard_gloo.py)."""
import os
import socket
import subprocess
import sys

import pytest

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_sharded_gemm_two_nccl_ranks(cuda):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port",
           str(_free_port()), os.path.join(ROOT, "tests", "shard_nccl_worker.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, cwd=ROOT, timeout=300,
                       env=dict(os.environ, NCCL_DEBUG="WARN"))
    log = r.stdout + r.stderr
    assert r.returncode == 0, log[-4000:]
    assert "OK rank 0 of 2" in log and "OK rank 1 of 2" in log, log[-4000:]
