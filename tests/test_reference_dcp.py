"""Sharded recovery checkpoints interchange with the reference's distributed trainer (``tnlm-dcp-v1``)
on two gloo ranks; skipped where the reference install under baseline/_ref is absent."""
import json
import os
import subprocess
import sys

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.path.join(os.path.dirname(HERE), "baseline", "_ref", "tnlm")


@pytest.mark.slow
@pytest.mark.skipif(not os.path.isdir(REF), reason="reference install absent")
@pytest.mark.parametrize("optimizer", ["adamw", "muon"])
def test_sharded_checkpoints_resume_across_frameworks(tmp_path, optimizer):
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", OMP_NUM_THREADS="1")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--standalone", "--local-addr", "127.0.0.1",
           "--nproc-per-node", "2", os.path.join(HERE, "dist_workers", "reference_dcp.py"), str(tmp_path), optimizer]
    out = subprocess.run(cmd, capture_output=True, text=True, timeout=900, env=env)
    assert out.returncode == 0, out.stdout[-3000:] + out.stderr[-5000:]
    assert "DCP_INTERCHANGE_OK" in out.stdout
    runs = json.loads((tmp_path / "losses.json").read_text())
    assert all(len(v) == 2 for v in runs.values())
    # a reference checkpoint continued here follows the reference's own continuation, and the reverse
    assert runs["ours-b"] == pytest.approx(runs["ref-b"], rel=1e-5)
    assert runs["ref-d"] == pytest.approx(runs["ours-d"], rel=1e-5)
    # both frameworks' first two updates agree as well (same data, same initialisation)
    assert runs["ours-c"] == pytest.approx(runs["ref-a"], rel=1e-5)
