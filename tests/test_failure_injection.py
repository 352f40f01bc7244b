"""Host-side failure injection on CPU ranks: a rank-local error, a corrupted shard, a departed rank,
a non-finite gradient on one rank and a full disk end as errors on every rank, never as a hang."""
import os
import subprocess
import sys

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


def _run(scenario, tmp_path, nproc=2):
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", OMP_NUM_THREADS="1")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--standalone", "--local-addr", "127.0.0.1",
           "--nproc-per-node", str(nproc), os.path.join(HERE, "dist_workers", "failure_injection.py"),
           scenario, str(tmp_path)]
    return subprocess.run(cmd, capture_output=True, text=True, timeout=180, env=env)


@pytest.mark.slow
@pytest.mark.parametrize("scenario,expected", [("phase", 2), ("corrupt", 2), ("dead_rank", 1), ("nonfinite", 2),
                                               ("disk_full", 2)])
def test_failures_reach_every_rank(scenario, expected, tmp_path):
    out = _run(scenario, tmp_path)
    assert out.stdout.count(f"SCENARIO_OK {scenario}") == expected, out.stdout[-2000:] + out.stderr[-3000:]
