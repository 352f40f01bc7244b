"""Batch branches of a serial checkpoint, sweep retention arithmetic, verified payload pruning and the
exact sweep-config export (CPU)."""
import copy
import hashlib
import json
import os

import pytest
import torch
import yaml

from helpers import TINY_MODEL
from tensor_train_ing_b200.batch_branch import BatchBranch
from tensor_train_ing_b200.config import Config, ModelConfig, TrainConfig
from tensor_train_ing_b200.models.model import TensorLM
from tensor_train_ing_b200.optim import make_optimizer
from tensor_train_ing_b200.hashing import canonical_sha256 as _digest
from tensor_train_ing_b200.sweep_config import export_sweep_config
from tensor_train_ing_b200.sweep_retention import (intermediate_payload, reject_symlink_chain, retention_forecast,
                                                   unlink_payload)


def _cfg(**train):
    return Config(model=ModelConfig(**TINY_MODEL),
                  train=TrainConfig(global_prediction_tokens_per_update=64, rung_total_tokens=10_000, lr=0.01,
                                    aux_adamw_lr=0.002, **train))


# --------------------------------------------------------------------------------- batch branch
def test_branch_config_scales_rates_and_sets_the_new_quota():
    cfg = _cfg()
    branch = BatchBranch.request(cfg, batch_tokens=128, lr_scale=2.0, resume="parent", context_fork=False,
                                 cooldown_steps=None)
    child = branch.child_config(cfg)
    assert child.train.global_prediction_tokens_per_update == 128
    assert child.train.lr == pytest.approx(0.02) and child.train.aux_adamw_lr == pytest.approx(0.004)
    assert cfg.train.lr == 0.01  # the parent config is untouched
    assert branch.record() == {"old_batch_tokens": 64, "new_batch_tokens": 128, "lr_scale": 2.0}
    assert BatchBranch.request(cfg, batch_tokens=None, lr_scale=None, resume=None, context_fork=False,
                               cooldown_steps=None) is None
    for bad in (dict(batch_tokens=64, lr_scale=2.0), dict(batch_tokens=128, lr_scale=0.0),
                dict(batch_tokens=128, lr_scale=float("inf")), dict(batch_tokens=128, lr_scale=None)):
        with pytest.raises(ValueError):
            BatchBranch.request(cfg, resume="parent", context_fork=False, cooldown_steps=None, **bad)
    with pytest.raises(ValueError):  # only from a constant schedule without a cooldown
        BatchBranch.request(cfg, batch_tokens=128, lr_scale=2.0, resume="p", context_fork=False, cooldown_steps=10)


def test_parent_must_be_past_warmup_and_before_its_horizon():
    child = _cfg()
    ok = {"progress": {"warmup_steps": 100, "scheduler_step": 150, "tokens": 5000, "steps": 150}}
    BatchBranch.check_parent(ok, child)
    for change in ({"scheduler_step": 50}, {"tokens": 10_000}, {"cooldown_start_tokens": 1}):
        bad = copy.deepcopy(ok)
        bad["progress"].update(change)
        with pytest.raises(ValueError):
            BatchBranch.check_parent(bad, child)


def test_apply_branch_scales_every_group_and_records_history():
    torch.manual_seed(0)
    model = TensorLM(ModelConfig(**TINY_MODEL))
    cfg = _cfg(optimizer="muon")
    opt = make_optimizer(model, cfg.train)
    before = [(g["lr"], g.get("base_lr")) for g in opt.param_groups]
    branch = BatchBranch.request(cfg, batch_tokens=32, lr_scale=0.5, resume="p", context_fork=False,
                                 cooldown_steps=None)
    child = branch.child_config(cfg)

    class Sampler:
        def state_dict(self):
            return {"cursor": 7}

    progress = {"tokens": 640, "steps": 10}
    branch.apply(opt, Sampler(), progress, cfg, child, {"path": "p"})
    for (lr, base), g in zip(before, opt.param_groups):
        assert g["lr"] == pytest.approx(0.5 * lr)
        assert g["base_lr"] == pytest.approx(0.5 * (base if base is not None else lr))
    entry = progress["batch_history"][-1]
    assert entry["source"] == "batch_branch" and entry["batch_tokens"] == 32 and entry["source_sampler"] == {"cursor": 7}
    assert progress["batch_history"][0]["source"] == "legacy_unknown"


# ------------------------------------------------------------------------------ sweep retention
def test_intermediate_payload_names():
    assert intermediate_payload("milestone-00001000/state.pt")
    assert intermediate_payload("recovery-00000010/state.pt")
    for name in ("final/state.pt", "milestone-/state.pt", "/milestone-1/state.pt", "a/milestone-1/state.pt",
                 "milestone-1/manifest.json"):
        assert not intermediate_payload(name)


def test_retention_forecast_keeps_initial_and_final_of_finished_candidates():
    plan = {"required_additional_bytes": 100, "per_checkpoint_estimate_bytes": 10,
            "count_breakdown": {"initial": 1, "final": 1, "milestones": 8}}
    runs = [{"name": n, "parent_storage_plan": plan, "cooldown_storage_plan": None} for n in ("a", "b", "c")]
    out = retention_forecast(runs)
    assert [r["new_prior_retained_bytes"] for r in out["candidates"]] == [0, 20, 40]
    assert out["required_additional_bytes"] == 140 and out["new_final_retained_bytes"] == 60
    done = retention_forecast(runs, completed_stages=["a/parent"])
    assert done["candidates"][0]["new_active_full_peak_bytes"] == 0


def test_verified_unlink_refuses_changed_payloads_and_symlinks(tmp_path):
    stage = tmp_path / "stage"
    (stage / "milestone-1").mkdir(parents=True)
    payload = stage / "milestone-1" / "state.pt"
    payload.write_bytes(b"weights")
    expected = {"bytes": 7, "sha256": hashlib.sha256(b"weights").hexdigest()}
    with pytest.raises(ValueError):
        unlink_payload(stage, "milestone-1/state.pt", {"bytes": 7, "sha256": "0" * 64})
    assert payload.exists()
    assert unlink_payload(stage, "milestone-1/state.pt", expected) is True
    assert not payload.exists()
    assert unlink_payload(stage, "milestone-1/state.pt", expected) is False  # already gone: a resumed prune
    with pytest.raises(ValueError):
        unlink_payload(stage, "../escape/state.pt", expected)
    target = tmp_path / "elsewhere"
    target.mkdir()
    os.symlink(target, stage / "recovery-2")
    with pytest.raises(ValueError):
        reject_symlink_chain(stage, stage / "recovery-2" / "state.pt")


# ----------------------------------------------------------------------------- sweep config export
def test_export_sweep_config_round_trips_the_recorded_config(tmp_path):
    config = {"model": {"layers": 2, "d_model": 32}, "train": {"lr": 0.01}}
    identity = {"version": 1, "trajectories": [{"name": "cand-a", "config": config, "config_sha256": _digest(config)}]}
    (tmp_path / "sweep.json").write_text(json.dumps({"identity": identity, "identity_sha256": _digest(identity)}))
    text = export_sweep_config(tmp_path, "cand-a")
    assert yaml.safe_load(text) == config and "provenance" in text
    with pytest.raises(ValueError):
        export_sweep_config(tmp_path, "missing")
    identity["trajectories"][0]["config"]["train"]["lr"] = 1.0  # tampered without updating checksums
    (tmp_path / "sweep.json").write_text(json.dumps({"identity": identity, "identity_sha256": _digest(identity)}))
    with pytest.raises(ValueError):
        export_sweep_config(tmp_path, "cand-a")


def test_sweep_plan_freezes_each_candidate_and_totals_the_projections(config):
    """Candidates are laid over the base config section by section, frozen with their digests, and
    their projected storage is summed; nothing is run or written."""
    from tensor_train_ing_b200.search import overlay, plan_sweep
    cands = [{"name": "base", "overrides": {}},
             {"name": "lr2x", "overrides": {"train": {"lr": 0.02}}},
             {"name": "wide", "overrides": {"model": {"d_model": 16}}}]
    plan = plan_sweep(config, cands)
    assert plan["candidate_count"] == 3 and [r["name"] for r in plan["runs"]] == ["base", "lr2x", "wide"]
    by = {r["name"]: r for r in plan["runs"]}
    assert by["lr2x"]["config"]["train"]["lr"] == 0.02 and by["base"]["config"]["train"]["lr"] == config.train.lr
    assert by["wide"]["config"]["model"]["d_model"] == 16
    assert len({r["config_sha256"] for r in plan["runs"]}) == 3
    assert plan["required_additional_bytes"] == sum(r["plan"]["checkpoint_storage_plan"]["required_additional_bytes"]
                                                    for r in plan["runs"])
    assert plan_sweep(config, cands)["runs"][1]["config_sha256"] == by["lr2x"]["config_sha256"]  # deterministic
    assert overlay({"a": {"b": 1, "c": 2}}, {"a": {"c": 3}}) == {"a": {"b": 1, "c": 3}}


@pytest.mark.parametrize("bad", [
    [],
    [{"name": "x"}],
    [{"name": "x", "overrides": {}, "extra": 1}],
    [{"name": "../up", "overrides": {}}],
    [{"name": "x", "overrides": {}}, {"name": "x", "overrides": {}}],
    [{"name": "x", "overrides": {"optimizer": {"lr": 1}}}],
    [{"name": "x", "overrides": {"train": 3}}],
    [{"name": "x", "overrides": {"model": {"layers": {"deep": 1}}}}],
])
def test_sweep_plan_refuses_malformed_candidates(config, bad):
    from tensor_train_ing_b200.search import plan_sweep
    with pytest.raises(ValueError):
        plan_sweep(config, bad)
