"""The sequence-sharded scan across GPUs over NCCL (two ranks and up), against
the unsplit scan.  Needs at least two GPUs; skipped otherwise."""
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_sequence_sharded_scan_over_nccl():
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs two GPUs")
    ranks = min(n, 8)
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", f"--nproc-per-node={ranks}", "--master-addr", "127.0.0.1",
           "--master-port", str(_free_port()), os.path.join(HERE, "seqshard_nccl_worker.py")]
    r = subprocess.run(cmd, capture_output=True, text=True, cwd=os.path.dirname(HERE))
    assert r.returncode == 0, r.stdout[-4000:] + r.stderr[-4000:]
