"""Distributed trainer on CPU ranks (gloo): exact resume replay and agreement with the serial trainer."""
import json
import os
import subprocess
import sys

import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _torchrun(worker, nproc, *args, timeout=600):
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", OMP_NUM_THREADS="1")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--standalone", "--local-addr", "127.0.0.1",
           "--nproc-per-node", str(nproc), os.path.join(HERE, "dist_workers", worker), *args]
    return subprocess.run(cmd, capture_output=True, text=True, timeout=timeout, env=env)


@pytest.mark.slow
@pytest.mark.parametrize("mode", ["replicated", "shard", "lagged", "taper", "cosine", "muon", "qkclip",
                                  "qkclip-shard"])
def test_two_rank_training_replays_and_matches_serial(tmp_path, mode):
    out = _torchrun("train_replay.py", 2, str(tmp_path), mode)
    assert out.returncode == 0, out.stdout[-3000:] + out.stderr[-4000:]
    assert "REPLAY_OK" in out.stdout
    sys.path.insert(0, os.path.join(HERE, "dist_workers"))
    from train_replay import config  # noqa: E402

    from tensor_train_ing_b200.train import train_run
    torch.set_num_threads(1)
    cfg = config(tmp_path, mode)
    cfg.raw["project"]["spend_ledger"] = str(tmp_path / "serial-spend.json")
    serial = train_run(cfg, tmp_path / "serial", max_steps=4, max_seconds=300, device="cpu")
    serial_losses = [json.loads(x)["loss"] for x in (tmp_path / "serial" / "metrics.jsonl").read_text().splitlines()]
    dist_losses = json.loads((tmp_path / "distributed_losses.json").read_text())
    assert serial["progress"]["tokens"] == 48
    if mode == "lagged":  # collective calibration reproduces the serial statistics
        assert serial["progress"]["calibration"]["tokens"] > 0
    if mode.startswith("qkclip"):
        # The serial trainer clips from its last micro-batch, the ranks from the maximum over their own
        # last micro-batches: the first update (before any clip) and its bound over every row agree,
        # the later ones need not.  The worker has checked that the ranks' replicated weights agree
        # (the checkpoint refuses otherwise) and that a resumed run replays the clipped one bitwise.
        rows = {name: [json.loads(x) for x in (tmp_path / name / "metrics.jsonl").read_text().splitlines()]
                for name in ("serial", "full")}
        for name, got in rows.items():  # a report every update; the first clips (later bounds sit near tau)
            assert all("qk_clip" in r and r["score_bound_max"] > 0 for r in got), name
            assert got[0]["qk_clip"]["clipped_heads"] > 0, name
        assert rows["serial"][0]["score_bound_max"] == pytest.approx(rows["full"][0]["score_bound_max"], rel=1e-5)
        assert serial_losses[0] == pytest.approx(dist_losses[0], rel=1e-5)
        return
    assert serial_losses == pytest.approx(dist_losses, rel=1e-5)
    s = torch.load(tmp_path / "serial" / "final" / "state.pt", weights_only=False)["model"]
    d = torch.load(tmp_path / "full" / "final-weights" / "state.pt", weights_only=False)["model"]
    for k in s:
        torch.testing.assert_close(s[k], d[k], rtol=1e-4, atol=1e-5)


@pytest.mark.slow
def test_two_rank_context_fork_is_recorded_and_deterministic(tmp_path):
    out = _torchrun("context_fork.py", 2, str(tmp_path))
    assert out.returncode == 0, out.stdout[-3000:] + out.stderr[-4000:]
    assert "FORK_OK" in out.stdout
