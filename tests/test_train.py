"""Serial trainer integration on CPU (tiny model, fixture dataset)."""
import copy
import math
import json

import pytest
import torch

from helpers import state
from tensor_train_ing_b200.budget import SpendLedger
from tensor_train_ing_b200.checkpoint import load_checkpoint
from tensor_train_ing_b200.models.model import TensorLM
from tensor_train_ing_b200.train import train_run


def _cfg(config, **train):
    cfg = copy.deepcopy(config)
    for k, v in train.items():
        setattr(cfg.train, k, v)
    return cfg


def test_interrupted_training_exact_replay(config, tmp_path):
    cfg = _cfg(config, deterministic=True)
    full = train_run(cfg, tmp_path / "full", max_steps=4, max_seconds=120, device="cpu")
    first = train_run(cfg, tmp_path / "a", max_steps=2, max_seconds=120, device="cpu")
    resumed = train_run(cfg, tmp_path / "b", max_steps=2, max_seconds=120, device="cpu", resume=first["checkpoint"])
    assert resumed["progress"]["steps"] == full["progress"]["steps"] == 4
    a, b = state(tmp_path / "full" / "final"), state(tmp_path / "b" / "final")
    for k, v in a["model"].items():
        assert torch.equal(v, b["model"][k]), k
    assert a["progress"]["tokens"] == b["progress"]["tokens"]


def test_dry_run_returns_plan_without_writing(config, tmp_path):
    cfg = copy.deepcopy(config)
    cfg.raw["project"]["dry_run"] = True
    plan = train_run(cfg, tmp_path / "dry", max_steps=1, max_seconds=1, device="cpu")
    assert plan["dry_run"] is True
    assert not (tmp_path / "dry").exists()


def test_result_records_progress_metrics_and_billing(config, tmp_path):
    r = train_run(config, tmp_path / "run", max_steps=3, max_seconds=120, device="cpu")
    assert r["progress"]["steps"] == 3
    assert r["progress"]["tokens"] == 3 * config.train.global_prediction_tokens_per_update
    rows = [json.loads(x) for x in (tmp_path / "run" / "metrics.jsonl").read_text().splitlines()]
    assert len(rows) >= 3 and all("loss" in x for x in rows if x.get("kind", "train") == "train")
    led = json.loads((tmp_path / "spend.json").read_text())
    assert any(run["status"] == "complete" for run in led["runs"].values())


def test_cooldown_forks_and_resumes_schedule(config, tmp_path):
    parent = train_run(config, tmp_path / "p", max_steps=2, max_seconds=120, device="cpu")
    cool = train_run(config, tmp_path / "c", max_steps=5, max_seconds=120, device="cpu",
                     resume=parent["checkpoint"], cooldown_steps=3)
    assert cool["training_descriptor"]["cooldown_status"] == "cooled"
    assert cool["progress"]["steps"] == 5


def test_resume_rejects_model_change(config, tmp_path):
    parent = train_run(config, tmp_path / "p", max_steps=1, max_seconds=120, device="cpu")
    other = copy.deepcopy(config)
    other.model.d_mlp = 16
    with pytest.raises(Exception):
        train_run(other, tmp_path / "x", max_steps=1, max_seconds=120, device="cpu", resume=parent["checkpoint"])


def test_checkpoint_loads_into_fresh_model(config, tmp_path):
    r = train_run(config, tmp_path / "run", max_steps=2, max_seconds=120, device="cpu")
    m = TensorLM(config.model)
    payload = load_checkpoint(r["checkpoint"], m, restore_rng=False, map_location="cpu")
    assert payload["progress"]["steps"] == 2
    saved = state(tmp_path / "run" / "final")["model"]
    for k, v in m.state_dict().items():
        assert torch.equal(v, saved[k])


def test_run_budget_cap_rejects_launch(config, tmp_path):
    cfg = copy.deepcopy(config)
    cfg.raw["project"]["gpu_hourly_rate_usd"] = 1000.0
    with pytest.raises(Exception):
        train_run(cfg, tmp_path / "run", max_steps=1, max_seconds=3600, device="cpu", run_budget_usd=0.01)


def test_spend_ledger_reservations_and_reconcile(tmp_path):
    led = SpendLedger(tmp_path / "l.json", 100.0, 10.0)
    led.begin("a", 36.0, 3600.0, None)  # reserves $36 of the 90 usable dollars
    led.finish("a", 1.0, "complete")  # charges one second
    data = json.loads((tmp_path / "l.json").read_text())
    assert data["runs"]["a"]["status"] == "complete"
    assert data["runs"]["a"]["spent_usd"] == pytest.approx(0.01)
    with pytest.raises(ValueError):
        led.begin("b", 3600.0, 3600.0, None)  # $3600 exceeds the budget left


def test_lagged_training_calibrates_before_the_first_update_and_replays(config, tmp_path):
    """The lagged package: site-by-site calibration on the calibration split before step 1, one
    committed statistic per update, and an exact resume across an interruption."""
    cfg = copy.deepcopy(config)
    cfg.model.normalization = "lagged"
    cfg.model.final_normalization = "lagged"
    full = train_run(cfg, tmp_path / "full", max_steps=3, max_seconds=120, device="cpu")
    cal = full["progress"]["calibration"]
    assert cal and cal.get("tokens", 0) > 0
    state = torch.load(tmp_path / "full" / "final" / "state.pt", weights_only=False)["model"]
    flags = [v for k, v in state.items() if k.endswith(".calibrated")]
    assert flags and all(bool(v) for v in flags)
    first = train_run(cfg, tmp_path / "a", max_steps=1, max_seconds=120, device="cpu")
    resumed = train_run(cfg, tmp_path / "b", max_steps=2, max_seconds=120, device="cpu", resume=first["checkpoint"])
    a = torch.load(tmp_path / "full" / "final" / "state.pt", weights_only=False)["model"]
    b = torch.load(tmp_path / "b" / "final" / "state.pt", weights_only=False)["model"]
    for k in a:
        assert torch.equal(a[k], b[k]), k
    assert resumed["progress"]["steps"] == full["progress"]["steps"] == 3


@pytest.mark.parametrize("package", ["branch_rms", "sandwich_rms", "group_rms", "spectral_rms", "taper"])
def test_every_normalization_package_trains_and_reloads(config, tmp_path, package):
    cfg = copy.deepcopy(config)
    cfg.model.normalization = package
    if package == "taper":
        cfg.model.final_normalization = "taper"
        cfg.train.taper_end_fraction = 1.0
        cfg.train.rung_total_tokens = 300 * cfg.train.global_prediction_tokens_per_update  # gate ends after warm-up
    r = train_run(cfg, tmp_path / "run", max_steps=2, max_seconds=120, device="cpu")
    rows = [json.loads(x) for x in (tmp_path / "run" / "metrics.jsonl").read_text().splitlines()]
    assert len(rows) == 2 and all(math.isfinite(x["loss"]) for x in rows)
    model = TensorLM(cfg.model)
    load_checkpoint(r["checkpoint"], model, restore_rng=False, map_location="cpu")


@pytest.mark.parametrize("source", ["probe", "batch_bound"])
def test_qk_clip_during_training_records_its_report(config, tmp_path, source):
    cfg = copy.deepcopy(config)
    cfg.train.qk_clip_tau = 1e-3  # far below any score: every head is clipped
    cfg.train.qk_clip_every_steps = 1
    cfg.train.qk_clip_source = source
    train_run(cfg, tmp_path / "run", max_steps=2, max_seconds=120, device="cpu")
    rows = [json.loads(x) for x in (tmp_path / "run" / "metrics.jsonl").read_text().splitlines()]
    clips = [x["qk_clip"] for x in rows if "qk_clip" in x]
    assert clips and all(c["clipped_heads"] > 0 for c in clips)
    if source == "batch_bound":
        assert all(x.get("score_bound_max", 0) > 0 for x in rows)


def test_context_fork_extends_the_context_and_records_history(config, tmp_path):
    parent = train_run(config, tmp_path / "p", max_steps=2, max_seconds=120, device="cpu")
    child_cfg = copy.deepcopy(config)
    child_cfg.raw["data"]["context"] = 6
    with pytest.raises(ValueError):  # a context change needs the explicit fork
        train_run(child_cfg, tmp_path / "x", max_steps=1, max_seconds=120, device="cpu", resume=parent["checkpoint"])
    child = train_run(child_cfg, tmp_path / "c", max_steps=2, max_seconds=120, device="cpu",
                      resume=parent["checkpoint"], context_fork=True)
    hist = child["progress"]["context_history"]
    assert [h["context"] for h in hist] == [4, 6]
    assert child["progress"]["steps"] == 4


def test_batch_branch_after_warmup_scales_rates_and_quota(config, tmp_path):
    cfg = copy.deepcopy(config)
    cfg.train.rung_total_tokens = 7 * 400
    parent = train_run(cfg, tmp_path / "p", max_steps=101, max_seconds=600, device="cpu")
    early = train_run(cfg, tmp_path / "e", max_steps=1, max_seconds=120, device="cpu")
    with pytest.raises(ValueError):  # the parent must be past its warm-up
        train_run(cfg, tmp_path / "x", max_steps=1, max_seconds=120, device="cpu", resume=early["checkpoint"],
                  batch_tokens=14, lr_scale=2.0)
    child = train_run(cfg, tmp_path / "c", max_steps=2, max_seconds=120, device="cpu", resume=parent["checkpoint"],
                      batch_tokens=14, lr_scale=2.0)
    last = child["progress"]["batch_history"][-1]
    assert last["source"] == "batch_branch" and last["batch_tokens"] == 14 and last["lr_scale"] == 2.0
    rows = [json.loads(x) for x in (tmp_path / "c" / "metrics.jsonl").read_text().splitlines()]
    assert all(r["prediction_tokens"] == 14 for r in rows)
    assert rows[0]["lr"] == pytest.approx(2 * cfg.train.lr)


def test_cosine_schedule_follows_its_multiplier(config, tmp_path):
    from tensor_train_ing_b200.schedules import schedule_multiplier
    cfg = copy.deepcopy(config)
    cfg.train.schedule = "cosine"
    cfg.train.rung_total_tokens = 7 * 150
    train_run(cfg, tmp_path / "run", max_steps=3, max_seconds=120, device="cpu")
    rows = [json.loads(x) for x in (tmp_path / "run" / "metrics.jsonl").read_text().splitlines()]
    for k, r in enumerate(rows):
        assert r["lr"] == pytest.approx(cfg.train.lr * schedule_multiplier(k, 150, schedule="cosine"))


def test_metrics_rows_carry_progress_rate_and_cost(config, tmp_path):
    """Each update row records the step, the cumulative tokens (one quota per update), the loss, the
    learning rate, the elapsed run time, the billed dollars at the configured rate and the token rate
    since the previous row; steps and times only grow."""
    cfg = copy.deepcopy(config)
    cfg.raw["project"]["gpu_hourly_rate_usd"] = 3.6
    train_run(cfg, tmp_path / "run", max_steps=4, max_seconds=120, device="cpu")
    rows = [json.loads(x) for x in (tmp_path / "run" / "metrics.jsonl").read_text().splitlines()]
    rows = [r for r in rows if r.get("kind", "train") == "train"]
    assert [r["step"] for r in rows] == [1, 2, 3, 4]
    quota = cfg.train.global_prediction_tokens_per_update
    assert [r["tokens"] for r in rows] == [quota * (i + 1) for i in range(4)]
    times = [r["run_elapsed_seconds"] for r in rows]
    assert times == sorted(times) and times[0] > 0
    for r in rows:
        assert r["loss"] > 0 and r["lr"] >= 0 and r["tokens_per_second"] > 0
        assert r["run_billed_usd"] == pytest.approx(r["run_elapsed_seconds"] * 3.6 / 3600)
