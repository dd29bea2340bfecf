"""Multi-GPU decode with the gather fused into the decode kernels (K5):
two to four ranks, one process per GPU (tests/gather_worker.py).  Skipped
when fewer than two GPUs are visible."""
from __future__ import annotations

import os
import socket
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.gpu
def test_gather_matches_per_rank_results():
    import torch
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs two GPUs")
    world = 4 if n >= 4 else 2
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", f"--nproc-per-node={world}", "--master-addr", "127.0.0.1",
           "--master-port", str(_free_port()), os.path.join(ROOT, "tests", "gather_worker.py")]
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=400)
    out = r.stdout + r.stderr
    assert r.returncode == 0, out[-4000:]
    for rank in range(world):
        assert f"RANK {rank} OK" in out, out[-4000:]
