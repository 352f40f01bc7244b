"""The command line on CPU: the reference's subcommands against a tiny fixture dataset."""
import json

import pytest
import torch
import yaml

from helpers import FixtureTokenizer
from tensor_train_ing_b200.cli import main
from tensor_train_ing_b200.data import prepare_data


@pytest.fixture
def setup(tmp_path):
    torch.set_num_threads(1)
    src = tmp_path / "src.jsonl"
    src.write_text("".join(json.dumps({"id": f"doc-{i}", "text": f"text number {i} " * 3}) + "\n" for i in range(60)))
    manifest = prepare_data(tmp_path / "data", source_jsonl=src, revision="offline-v1", tokenizer=FixtureTokenizer(),
                            split_fractions={"train": .6, "val": .3, "test": 0., "calibration": .1})
    cfg = {"model": {"layers": 1, "d_model": 8, "heads": 1, "d_key": 4, "d_value": 4, "d_mlp": 12,
                     "padded_vocab": 50257},
           "train": {"compile": False, "bf16_compute": False, "global_prediction_tokens_per_update": 20,
                     "rung_total_tokens": 200, "lr": 0.01},
           "data": {"manifest": str(manifest), "context": 16, "micro_batch_size": 2, "calibration_tokens": 8},
           "project": {"dry_run": False, "gpu_hourly_rate_usd": 0, "spend_ledger": str(tmp_path / "spend.json")}}
    path = tmp_path / "cfg.yaml"
    path.write_text(yaml.safe_dump(cfg))
    return path, tmp_path


def _run(capsys, *argv):
    assert main([str(a) for a in argv]) == 0
    return json.loads(capsys.readouterr().out)


def test_validate_and_plan(setup, capsys):
    cfg, tmp = setup
    v = _run(capsys, "validate_config", "--config", cfg, "--device", "cpu", "--run-dir", tmp / "x")
    assert v["parameters"]["total"] > 0 and v["checkpoint_disk_check"]["status"] == "ok"
    p = _run(capsys, "plan_search", "--config", cfg)
    assert p["planned_optimizer_steps"] == 10


def test_train_cooldown_evaluate_analyze_summarize(setup, capsys):
    cfg, tmp = setup
    r = _run(capsys, "train", "--config", cfg, "--run-dir", tmp / "run", "--max-steps", 3, "--max-seconds", 120,
             "--device", "cpu")
    assert r["progress"]["steps"] == 3
    c = _run(capsys, "cooldown", "--config", cfg, "--run-dir", tmp / "cool", "--max-steps", 2, "--max-seconds", 120,
             "--device", "cpu", "--resume", r["checkpoint"], "--cooldown-steps", 2)
    assert c["training_descriptor"]["cooldown_status"] == "cooled"
    e = _run(capsys, "evaluate", "--config", cfg, "--checkpoint", c["checkpoint"], "--out", tmp / "eval",
             "--max-seconds", 120, "--bootstrap-samples", 10)
    assert e["prediction_tokens"] > 0
    e2 = _run(capsys, "evaluate", "--config", cfg, "--checkpoint", r["checkpoint"], "--out", tmp / "eval2",
              "--max-seconds", 120, "--bootstrap-samples", 10)
    cmp = _run(capsys, "compare_evaluations", "--left", tmp / "eval2" / "evaluation.json",
               "--right", tmp / "eval" / "evaluation.json", "--out", tmp / "cmp", "--bootstrap-samples", 10)
    assert cmp["delta_ce_right_minus_left"] == pytest.approx(e["ce"] - e2["ce"])
    a = _run(capsys, "analyze", "--config", cfg, "--checkpoint", c["checkpoint"], "--out", tmp / "ana",
             "--batches", 1)
    assert a["evaluation_provenance"]["frozen_state"]["unchanged"]
    s = _run(capsys, "summarize", "--run-dirs", tmp / "run", tmp / "cool", "--out", tmp / "summary")
    assert s["runs"] == 2 and "loss-vs-tokens.svg" in s["artifacts"]
    spend = _run(capsys, "record_spend", "--config", cfg, "--charge-id", "storage", "--usd", 1.5, "--stage", "Reserve",
                 "--description", "disk")
    assert spend["spent_usd"] == 1.5
    with pytest.raises(ValueError, match="unresolved"):  # only unresolved runtime entries reconcile
        main(["reconcile", "--ledger", str(tmp / "spend.json"), "--run-id", str((tmp / "run").resolve())])


def test_sweep_and_export(setup, capsys):
    cfg, tmp = setup
    cands = tmp / "cands.yaml"
    cands.write_text(yaml.safe_dump([{"name": "base", "overrides": {}},
                                     {"name": "lr2", "overrides": {"train": {"lr": 0.02}}}]))
    out = _run(capsys, "sweep", "--config", cfg, "--candidates", cands, "--out", tmp / "sweep",
               "--max-seconds", 120, "--evaluation-max-seconds", 120, "--device", "cpu", "--bootstrap-samples", 10)
    assert out["status"] == "complete"
    assert len(out["identity"]["trajectories"]) == 2
    assert main(["sweep-config", "--sweep", str(tmp / "sweep"), "--candidate", "lr2"]) == 0
    text = capsys.readouterr().out
    assert "lr: 0.02" in text
    again = _run(capsys, "sweep", "--config", cfg, "--candidates", cands, "--out", tmp / "sweep",
                 "--max-seconds", 120, "--evaluation-max-seconds", 120, "--device", "cpu", "--bootstrap-samples", 10)
    assert again["status"] == "complete"  # every stage reused after hash verification


def test_prepare_mechanisms(tmp_path, capsys):
    r = _run(capsys, "prepare_mechanisms", "--out", tmp_path / "tasks", "--seed", 3, "--train-examples", 8,
             "--validation-examples", 8)
    assert r["manifest"]


def test_profile_command_reports_post_warmup_steps_and_writes_a_trace(setup, capsys):
    cfg, tmp = setup
    r = _run(capsys, "profile", "--config", cfg, "--run-dir", tmp / "prof", "--steps", 3, "--warmup-steps", 1,
             "--trace-steps", 1, "--max-seconds", 120, "--device", "cpu")
    assert (r["completed_timed_steps"], r["warmup_steps"], r["completed_total_steps"]) == (3, 1, 4)
    assert r["timed_prediction_tokens"] == 3 * 20  # three timed updates of 20 scored tokens each
    assert r["stop_reason"] == "max_steps" and r["prediction_tokens_per_second"] > 0
    assert (tmp / "prof" / "profile.json").exists() and (tmp / "prof" / "metrics.jsonl").exists()


def test_branch_refuses_a_parent_still_in_warmup(setup, capsys):
    cfg, tmp = setup
    r = _run(capsys, "train", "--config", cfg, "--run-dir", tmp / "run", "--max-steps", 2, "--max-seconds", 120,
             "--device", "cpu")
    with pytest.raises(ValueError):
        main(["branch", "--config", str(cfg), "--run-dir", str(tmp / "b"), "--max-steps", "1", "--max-seconds", "60",
              "--device", "cpu", "--resume", r["checkpoint"], "--batch-tokens", "40", "--lr-scale", "2.0"])
    assert not (tmp / "b" / "result.json").exists()


def test_compare_seed_pairs_command_validates_before_writing(setup, capsys):
    cfg, tmp = setup
    pairs = tmp / "pairs.json"
    pairs.write_text(json.dumps([{"seed": 1, "left": "a.json", "right": "b.json"}]))
    with pytest.raises(ValueError, match="two"):
        main(["compare_seed_pairs", "--pairs", str(pairs), "--out", str(tmp / "rep")])
    assert not (tmp / "rep").exists()


def test_every_subcommand_documents_its_flags():
    """The reference's command surface: the parser has exactly the reference's nineteen subcommands,
    and each parses --help (exit 0)."""
    import argparse
    import contextlib
    import io

    from tensor_train_ing_b200.cli import _parser
    parser = _parser()
    actions = [a for a in parser._actions if isinstance(a, argparse._SubParsersAction)]
    names = sorted(actions[0].choices)
    assert names == sorted(["analyze", "branch", "check_math", "compare_evaluations", "compare_seed_pairs",
                            "cooldown", "evaluate", "evaluate_mechanisms", "plan_search", "prepare_data",
                            "prepare_mechanisms", "profile", "reconcile", "record_spend", "summarize", "sweep",
                            "sweep-config", "train", "validate_config"])
    for name in names:
        out = io.StringIO()
        with contextlib.redirect_stdout(out), pytest.raises(SystemExit) as exit_info:
            parser.parse_args([name, "--help"])
        assert exit_info.value.code == 0 and "usage:" in out.getvalue(), name
