"""Context forks in the serial trainer, on CPU (beyond the basic fork in test_train):

* a forked run interrupted and resumed equals the uninterrupted fork bit for bit;
* under the cosine schedule a fork keeps the parent's global horizon: its rates continue the
  parent's multiplier from the parent's scheduler step;
* refused changes (a smaller or equal context, a fork without a parent, a malformed flag) fail
  before the run reserves any budget or creates its directory; a dry run reads no parent, so it
  refuses the flag errors and leaves the context check to the real run ("pending");
* the fork's history records the parent and the sampler position it left from, and a fork of a
  fork appends to the history.
"""
import copy
import json

import pytest
import torch

from helpers import state
from tensor_train_ing_b200.schedules import schedule_multiplier
from tensor_train_ing_b200.train import train_run


def _rows(path):
    return [json.loads(x) for x in (path / "metrics.jsonl").read_text().splitlines()]


def _with_context(cfg, context):
    out = copy.deepcopy(cfg)
    out.raw["data"]["context"] = context
    return out


def test_a_forked_run_resumes_exactly(config, tmp_path):
    cfg = copy.deepcopy(config)
    cfg.train.deterministic = True
    parent = train_run(cfg, tmp_path / "p", max_steps=2, max_seconds=120, device="cpu")
    longer = _with_context(cfg, 8)
    whole = train_run(longer, tmp_path / "whole", max_steps=4, max_seconds=120, device="cpu",
                      resume=parent["checkpoint"], context_fork=True)
    first = train_run(longer, tmp_path / "first", max_steps=2, max_seconds=120, device="cpu",
                      resume=parent["checkpoint"], context_fork=True)
    second = train_run(longer, tmp_path / "second", max_steps=2, max_seconds=120, device="cpu",
                       resume=first["checkpoint"])  # same context now: a plain resume
    assert whole["progress"]["steps"] == second["progress"]["steps"] == 6
    a, b = state(tmp_path / "whole" / "final"), state(tmp_path / "second" / "final")
    for k, v in a["model"].items():
        assert torch.equal(v, b["model"][k]), k
    assert [r["loss"] for r in _rows(tmp_path / "whole")][2:] == [r["loss"] for r in _rows(tmp_path / "second")]
    assert second["progress"]["context_history"] == whole["progress"]["context_history"]


def test_a_cosine_fork_keeps_the_global_horizon(config, tmp_path):
    cfg = copy.deepcopy(config)
    cfg.train.schedule = "cosine"
    quota = cfg.train.global_prediction_tokens_per_update
    total = 150
    cfg.train.rung_total_tokens = quota * total
    parent = train_run(cfg, tmp_path / "p", max_steps=3, max_seconds=120, device="cpu")
    child = train_run(_with_context(cfg, 8), tmp_path / "c", max_steps=3, max_seconds=120, device="cpu",
                      resume=parent["checkpoint"], context_fork=True)
    assert child["progress"]["scheduler_step"] == 6
    for k, r in enumerate(_rows(tmp_path / "c")):
        assert r["lr"] == pytest.approx(cfg.train.lr * schedule_multiplier(3 + k, total, schedule="cosine"))


@pytest.mark.parametrize("dry_run", [False, True])
def test_refused_forks_fail_before_any_reservation(config, tmp_path, dry_run):
    parent = train_run(config, tmp_path / "p", max_steps=1, max_seconds=120, device="cpu")
    ledger = tmp_path / "spend.json"
    cfg = copy.deepcopy(config)
    cfg.raw["project"]["spend_ledger"] = str(ledger)
    cfg.raw["project"]["dry_run"] = dry_run
    before = ledger.read_bytes() if ledger.exists() else None
    cases = [(_with_context(cfg, 4), dict(resume=parent["checkpoint"], context_fork=True), "strictly increasing"),
             (_with_context(cfg, 2), dict(resume=parent["checkpoint"], context_fork=True), "strictly increasing"),
             (_with_context(cfg, 8), dict(context_fork=True), "parent"),
             (_with_context(cfg, 8), dict(resume=parent["checkpoint"], context_fork="yes"), "Boolean")]
    for i, (c, kw, message) in enumerate(cases):
        if dry_run and "resume" in kw and kw.get("context_fork") is True:
            plan = train_run(c, tmp_path / f"x{i}", max_steps=1, max_seconds=120, device="cpu", **kw)
            assert plan["parent_validation"] == "pending"
        else:
            with pytest.raises(ValueError, match=message):
                train_run(c, tmp_path / f"x{i}", max_steps=1, max_seconds=120, device="cpu", **kw)
        assert not (tmp_path / f"x{i}").exists()
    assert (ledger.read_bytes() if ledger.exists() else None) == before


def test_fork_history_records_the_parent_and_chains(config, tmp_path):
    parent = train_run(config, tmp_path / "p", max_steps=2, max_seconds=120, device="cpu")
    mid = train_run(_with_context(config, 6), tmp_path / "m", max_steps=1, max_seconds=120, device="cpu",
                    resume=parent["checkpoint"], context_fork=True)
    top = train_run(_with_context(config, 8), tmp_path / "t", max_steps=1, max_seconds=120, device="cpu",
                    resume=mid["checkpoint"], context_fork=True)
    hist = top["progress"]["context_history"]
    assert [h["context"] for h in hist] == [4, 6, 8]
    assert [h["source"] for h in hist] == ["fresh", "context_fork", "context_fork"]
    assert [h["start_step"] for h in hist] == [0, 2, 3]
    assert hist[1]["start_tokens"] == parent["progress"]["tokens"]
    assert all(h.get("parent") and h.get("source_sampler") for h in hist[1:])
