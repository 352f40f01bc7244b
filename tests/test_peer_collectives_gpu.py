"""Peer-memory collectives on 2 GPUs against NCCL (skipped with fewer than two GPUs)."""
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_peer_reduce_scatter_and_all_gather_match_nccl():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = ["timeout", "-k", "30", "600", sys.executable, "-m", "torch.distributed.run", "--standalone",
           "--local-addr", "127.0.0.1", "--nproc-per-node", "2", os.path.join(HERE, "dist_workers", "peer_collectives.py")]
    out = subprocess.run(cmd, capture_output=True, text=True, timeout=660, env=env)
    assert out.returncode == 0, out.stdout[-3000:] + out.stderr[-4000:]
    assert "PEER_OK" in out.stdout
