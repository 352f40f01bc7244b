"""Operational tools on CPU: throughput and regression checks, the scaling grid (plan, run, fit),
run audits and the trainer smoke."""
import json

import pytest
import torch
import yaml

from helpers import FixtureTokenizer
from tensor_train_ing_b200.data import prepare_data
from tensor_train_ing_b200.runbook import audit, scaling, smoke, throughput


def _metrics(path, rates):
    rows, t, tok = [], 0.0, 0
    for i, r in enumerate(rates, 1):
        t += 1.0
        tok += int(r)
        rows.append({"step": i, "tokens": tok, "run_elapsed_seconds": t, "prediction_tokens": int(r), "seconds": 1.0})
    path.parent.mkdir(parents=True, exist_ok=True)
    path.write_text("".join(json.dumps(x) + "\n" for x in rows))
    return path


def test_steady_rate_drop_ratio_and_regressions(tmp_path):
    m = _metrics(tmp_path / "a" / "parent" / "metrics.jsonl", [10] * 5 + [1000] * 45)
    assert throughput.steady_rate(m) == pytest.approx(1000)
    slow = _metrics(tmp_path / "b" / "metrics.jsonl", [1000] * 30 + [500] * 20)
    # recent: the last 10 rows at 500/s; steady: rows 26..50, 4 at 1000/s and 20 at 500/s over 24 s
    assert throughput.drop_ratio(slow, last=10) == pytest.approx(500 / ((4 * 1000 + 20 * 500) / 24), rel=1e-9)
    measured = throughput.rates([tmp_path])
    assert set(measured) == {"a", "b"}
    bad = throughput.regressions(measured, {"a": 1100.0, "b": 500.0}, tolerance=0.05)
    assert [r["run"] for r in bad] == ["a"]
    assert throughput.main([str(tmp_path), "--record", str(tmp_path / "base.json")]) == 0
    assert throughput.main([str(tmp_path), "--baseline", str(tmp_path / "base.json")]) == 0


def test_scaling_law_fit_recovers_a_known_law():
    law = {"E": 1.7, "A": 400.0, "B": 1200.0, "alpha": 0.34, "beta": 0.28}
    points = [(n, d, law["E"] + law["A"] / n ** law["alpha"] + law["B"] / d ** law["beta"])
              for n in (2e7, 5e7, 1e8, 3e8) for d in (1e9, 3e9, 1e10)]
    starts = [(5.0, 5.0, 0.5, 0.5, 0.5), (6.0, 7.0, 0.5, 0.3, 0.3), (10.0, 10.0, 0.0, 0.5, 0.5)]
    got = scaling.fit(points, starts=starts)
    # E trades off against B / D^beta over this range of D: the exponents and the fitted curve are tight
    assert got["alpha"] == pytest.approx(law["alpha"], rel=2e-2)
    assert got["beta"] == pytest.approx(law["beta"], rel=5e-2) and got["E"] == pytest.approx(law["E"], rel=5e-2)
    assert max(abs(got["E"] + got["A"] / n ** got["alpha"] + got["B"] / d ** got["beta"] - loss) / loss
               for n, d, loss in points) < 2e-3
    opt = scaling.compute_optimal(got, 1e21)
    assert 6 * opt["N_opt"] * opt["D_opt"] == pytest.approx(1e21, rel=1e-9)
    # the optimum beats its neighbours along the compute frontier
    def loss_at(n):
        d = 1e21 / 6 / n
        return got["E"] + got["A"] / n ** got["alpha"] + got["B"] / d ** got["beta"]
    assert loss_at(opt["N_opt"]) <= min(loss_at(opt["N_opt"] * 1.2), loss_at(opt["N_opt"] / 1.2))


@pytest.fixture
def dataset(tmp_path):
    src = tmp_path / "src.jsonl"
    src.write_text("".join(json.dumps({"id": f"d{i}", "text": f"document {i} " * 4}) + "\n" for i in range(60)))
    return prepare_data(tmp_path / "data", source_jsonl=src, revision="offline-v1", tokenizer=FixtureTokenizer(),
                        split_fractions={"train": .6, "val": .3, "test": 0., "calibration": .1})


def _base(dataset, tmp_path):
    return {"model": {"layers": 1, "d_model": 8, "heads": 1, "d_key": 4, "d_value": 4, "d_mlp": 12,
                      "padded_vocab": 50257},
            "train": {"compile": False, "bf16_compute": False, "global_prediction_tokens_per_update": 7, "lr": 0.01},
            "data": {"manifest": str(dataset), "context": 8, "micro_batch_size": 1},
            "project": {"dry_run": False, "gpu_hourly_rate_usd": 0, "spend_ledger": str(tmp_path / "spend.json")}}


def test_scaling_grid_plans_runs_and_resumes(dataset, tmp_path):
    torch.set_num_threads(1)
    grid = {"base": _base(dataset, tmp_path), "sizes": {"s8": {"model": {"d_model": 8}, "lr": 0.01}}}
    plan = scaling.plan_size(grid, "s8", tpps=(1e-4, 2e-4), out_root=tmp_path / "grid")
    assert plan["budgets"] == [77, 161] and plan["branch_tokens"] == {"77": 70, "161": 147}
    report = scaling.run_size(plan, device="cpu", max_seconds=300, bootstrap_samples=10)
    assert [b["tokens"] for b in report["budgets"]] == [77, 161]
    points = scaling.collect(tmp_path / "grid")
    assert sorted(p[1] for p in points) == [77.0, 161.0]
    again = scaling.run_size(plan, device="cpu", max_seconds=300)  # every stage is found finished
    assert again == report


def test_audits_flag_epoch_overreads_search_and_stability(tmp_path):
    manifest = tmp_path / "m.json"
    manifest.write_text(json.dumps({"tokens": {"train": 100}}))
    for name, seen in (("ok", 90), ("over", 250)):
        (tmp_path / name).mkdir()
        (tmp_path / name / "result.json").write_text(json.dumps({
            "progress": {"input_tokens_seen": seen},
            "training_descriptor": {"configuration": {"data": {"manifest": str(manifest)}}}}))
    found = audit.epoch_overreads([tmp_path])
    assert [r["epochs"] for r in found] == [2.5]
    for name, ce, norm in (("e1", 3.1, "pre_rms"), ("e2", 2.9, "pre_rms"), ("e3", 2.5, "lagged")):
        (tmp_path / name).mkdir()
        (tmp_path / name / "evaluation.json").write_text(json.dumps({
            "kind": "held_out_validation", "ce": ce, "prediction_tokens": 10,
            "training_descriptor": {"normalization": norm, "width": 8}}))
    rows = audit.find_runs([tmp_path], {"normalization": "pre_rms", "width": 8})
    assert [r["ce"] for r in rows] == [2.9, 3.1]
    metrics = tmp_path / "metrics.jsonl"
    metrics.write_text("".join(json.dumps({"step": i, "score_bound_max": v}) + "\n"
                               for i, v in enumerate([1.0, 1.1, 1.2, 5.0, 5.1], 1)))
    trace = audit.stability_trace(metrics, jump=2.0, absolute=5.05)
    assert [r["flags"] for r in trace] == [[], [], [], ["jump"], ["absolute"]]


def test_trainer_smoke_replays_and_evaluates(dataset, tmp_path):
    torch.set_num_threads(1)
    path = tmp_path / "run.yaml"
    doc = _base(dataset, tmp_path)
    doc["train"]["rung_total_tokens"] = 200
    path.write_text(yaml.safe_dump(doc))
    report = smoke.run_smoke(path, tmp_path / "smoke", steps=2, device="cpu", max_seconds=300, bootstrap_samples=10)
    assert report["status"] == "passed" and report["replay_bitwise_identical"]
    assert report["uninterrupted_losses"] == report["interrupted_losses"]
    assert report["evaluation_prediction_tokens"] > 0
