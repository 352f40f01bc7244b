"""Pruning a sweep's intermediate checkpoints (``run_sweep(..., prune_completed_intermediates=True)``)
on CPU, end to end:

* after a candidate is evaluated, its milestone payloads are deleted under the ledger's lock while
  the initial and final checkpoints, every manifest, the metrics and the results stay; the
  evaluation equals that of a sweep that kept everything;
* a prune interrupted between two deletions is journaled as planned and the next invocation
  finishes it without training or evaluating again;
* a slated payload or a retained artifact that changed after the plan was journaled, or a stage
  directory swapped for a symbolic link, stops the prune before any other deletion;
* a run in the spend ledger that still uses a slated checkpoint as its parent blocks the prune.
"""
import fcntl
import json
from pathlib import Path

import pytest
import torch

from helpers import FixtureTokenizer
from tensor_train_ing_b200 import sweep as sweep_module
from tensor_train_ing_b200.config import Config
from tensor_train_ing_b200.data import prepare_data
from tensor_train_ing_b200.sweep import run_sweep
from tensor_train_ing_b200.sweep_retention import intermediate_payload


@pytest.fixture
def cfg(tmp_path):
    import yaml
    torch.set_num_threads(1)
    src = tmp_path / "src.jsonl"
    src.write_text("".join(json.dumps({"id": f"doc-{i}", "text": f"text number {i} " * 3}) + "\n" for i in range(60)))
    manifest = prepare_data(tmp_path / "data", source_jsonl=src, revision="offline-v1", tokenizer=FixtureTokenizer(),
                            split_fractions={"train": .6, "val": .3, "test": 0., "calibration": .1})
    raw = {"model": {"layers": 1, "d_model": 8, "heads": 1, "d_key": 4, "d_value": 4, "d_mlp": 12,
                     "padded_vocab": 50257},
           "train": {"compile": False, "bf16_compute": False, "global_prediction_tokens_per_update": 20,
                     "rung_total_tokens": 200, "lr": 0.01},
           "data": {"manifest": str(manifest), "context": 16, "micro_batch_size": 2, "calibration_tokens": 8},
           "project": {"dry_run": False, "gpu_hourly_rate_usd": 0, "spend_ledger": str(tmp_path / "spend.json"),
                       "milestone_tokens": [40, 100], "keep_recovery_checkpoints": 0}}
    path = tmp_path / "cfg.yaml"
    path.write_text(yaml.safe_dump(raw))
    return Config.from_yaml(str(path))


def _sweep(cfg, out, *, prune=True, two=True):
    candidates = [{"name": "a", "overrides": {}}]
    if two:
        candidates.append({"name": "b", "overrides": {"train": {"lr": 0.02}}})
    return run_sweep(cfg, candidates, out, max_seconds=120, evaluation_max_seconds=120, device="cpu",
                     max_prediction_tokens=14, bootstrap_samples=5, prune_completed_intermediates=prune)


def _forbid_work(monkeypatch):
    def forbidden(*args, **kwargs):
        raise AssertionError("a completed stage ran again")
    for name in ("train_run", "evaluate_checkpoint", "compare_evaluations", "summarize_runs"):
        monkeypatch.setattr(sweep_module, name, forbidden)


@pytest.mark.slow
def test_prune_keeps_endpoints_and_evaluations(cfg, tmp_path, monkeypatch):
    kept = _sweep(cfg, tmp_path / "kept", prune=False)
    assert list((tmp_path / "kept").glob("*/parent/milestone-*/state.pt"))
    locked = []
    real_unlink = sweep_module.unlink_payload

    def unlink_under_lock(*args):
        with Path(str(cfg.raw["project"]["spend_ledger"]) + ".lock").open("a") as probe:
            with pytest.raises(BlockingIOError):  # the prune holds the ledger's admission lock
                fcntl.flock(probe, fcntl.LOCK_EX | fcntl.LOCK_NB)
        locked.append(args[1])
        return real_unlink(*args)
    monkeypatch.setattr(sweep_module, "unlink_payload", unlink_under_lock)
    out = tmp_path / "pruned"
    result = _sweep(cfg, out)
    assert kept["status"] == result["status"] == "complete" and locked
    for name in ("a", "b"):
        for phase in ("parent", "cooldown"):
            stage = out / name / phase
            assert (stage / "initial" / "state.pt").is_file() and (stage / "final" / "state.pt").is_file()
            assert (stage / "metrics.jsonl").is_file() and (stage / "result.json").is_file()
            assert not list(stage.glob("milestone-*/state.pt")) and not list(stage.glob("recovery-*/state.pt"))
        op = result["prune_operations"][name]
        assert op["status"] == "complete" and op["files"]
        assert op["original_payload_bytes"] == sum(f["bytes"] for f in op["files"].values())
        for rel, info in op["files"].items():
            assert intermediate_payload(info["artifact"]) and not (out / rel).exists()
            assert (out / rel).with_name("manifest.json").is_file()  # the manifest stays
        a = json.loads((tmp_path / "kept" / name / "evaluation" / "evaluation.json").read_text())
        b = json.loads((out / name / "evaluation" / "evaluation.json").read_text())
        assert a["ce"] == b["ce"] and a["model_sha256"] == b["model_sha256"]
    ledger = Path(cfg.raw["project"]["spend_ledger"]).read_bytes()
    monkeypatch.setattr(sweep_module, "unlink_payload", real_unlink)
    _forbid_work(monkeypatch)
    assert _sweep(cfg, out)["status"] == "complete"  # re-entry verifies, trains nothing, bills nothing
    assert Path(cfg.raw["project"]["spend_ledger"]).read_bytes() == ledger


def _interrupt_after_one_deletion(cfg, out, monkeypatch):
    real = sweep_module.unlink_payload
    calls = []

    def interrupted(*args):
        calls.append(args[1])
        if len(calls) == 2:
            raise RuntimeError("injected interruption between deletions")
        return real(*args)
    monkeypatch.setattr(sweep_module, "unlink_payload", interrupted)
    with pytest.raises(RuntimeError, match="injected interruption"):
        _sweep(cfg, out, two=False)
    monkeypatch.setattr(sweep_module, "unlink_payload", real)
    journal = json.loads((out / "sweep.json").read_text())
    op = journal["prune_operations"]["a"]
    assert op["status"] == "planned" and len(op["files"]) >= 2
    assert sum(not (out / rel).exists() for rel in op["files"]) == 1
    return op


@pytest.mark.slow
def test_interrupted_prune_finishes_without_retraining(cfg, tmp_path, monkeypatch):
    out = tmp_path / "sweep"
    op = _interrupt_after_one_deletion(cfg, out, monkeypatch)
    ledger = Path(cfg.raw["project"]["spend_ledger"]).read_bytes()

    def forbidden(*args, **kwargs):
        raise AssertionError("a billed stage ran again")
    # the summary had not run before the interruption; the billed stages must not run again
    monkeypatch.setattr(sweep_module, "train_run", forbidden)
    monkeypatch.setattr(sweep_module, "evaluate_checkpoint", forbidden)
    result = _sweep(cfg, out, two=False)
    assert result["status"] == "complete" and result["prune_operations"]["a"]["status"] == "complete"
    assert not any((out / rel).exists() for rel in op["files"])
    assert Path(cfg.raw["project"]["spend_ledger"]).read_bytes() == ledger


@pytest.mark.slow
@pytest.mark.parametrize("changed", ["slated payload", "retained result"])
def test_a_changed_file_stops_a_pending_prune(cfg, tmp_path, monkeypatch, changed):
    out = tmp_path / "sweep"
    op = _interrupt_after_one_deletion(cfg, out, monkeypatch)
    remaining = [out / rel for rel in op["files"] if (out / rel).exists()]
    target = remaining[0] if changed == "slated payload" else out / "a" / "parent" / "result.json"
    with target.open("ab") as fh:
        fh.write(b"tampered")
    before = {p: p.read_bytes() for p in remaining}
    _forbid_work(monkeypatch)
    with pytest.raises(ValueError):
        _sweep(cfg, out, two=False)
    assert all(p.exists() and p.read_bytes() == before[p] for p in remaining)  # nothing more was deleted
    assert json.loads((out / "sweep.json").read_text())["prune_operations"]["a"]["status"] == "planned"


@pytest.mark.slow
@pytest.mark.parametrize("redirect", ["stage", "candidate"])
def test_a_symlinked_directory_stops_a_pending_prune(cfg, tmp_path, monkeypatch, redirect):
    """A stage (or candidate) directory replaced by a link to a copy elsewhere: the prune refuses
    and deletes nothing outside the sweep."""
    out = tmp_path / "sweep"
    _interrupt_after_one_deletion(cfg, out, monkeypatch)
    moved = out / "a" / "parent" if redirect == "stage" else out / "a"
    elsewhere = tmp_path / "elsewhere"
    moved.rename(elsewhere)
    moved.symlink_to(elsewhere, target_is_directory=True)
    before = {p: p.read_bytes() for p in elsewhere.rglob("*") if p.is_file()}
    _forbid_work(monkeypatch)
    with pytest.raises(ValueError, match="symlink"):
        _sweep(cfg, out, two=False)
    assert {p: p.read_bytes() for p in elsewhere.rglob("*") if p.is_file()} == before


@pytest.mark.slow
def test_a_run_that_uses_a_slated_checkpoint_blocks_the_prune(cfg, tmp_path, monkeypatch):
    unlinked = []
    real_unlink, real_eval = sweep_module.unlink_payload, sweep_module.evaluate_checkpoint

    def count_unlink(*args):
        unlinked.append(args[1])
        return real_unlink(*args)

    def pin_after_evaluation(*args, **kwargs):
        report = real_eval(*args, **kwargs)
        ledger_path = Path(cfg.raw["project"]["spend_ledger"])
        ledger = json.loads(ledger_path.read_text())
        milestone = sorted((out / "a" / "parent").glob("milestone-*"))[0]
        ledger["runs"]["someone-else"] = {"status": "running", "reserved_usd": 1.0,
                                          "parent_checkpoint": str(milestone.resolve())}
        ledger_path.write_text(json.dumps(ledger))
        return report
    monkeypatch.setattr(sweep_module, "unlink_payload", count_unlink)
    monkeypatch.setattr(sweep_module, "evaluate_checkpoint", pin_after_evaluation)
    out = tmp_path / "sweep"
    with pytest.raises(ValueError, match="pins"):
        _sweep(cfg, out, two=False)
    assert not unlinked and list((out / "a" / "parent").glob("milestone-*/state.pt"))
