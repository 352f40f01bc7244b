"""Batch-size history in the training evidence of an evaluation report (``evaluate._training_descriptor``
and ``_training_comparison``), on hand-built checkpoint payloads:

* a complete history keeps each segment's quota, rates, start and source, and drops the artifact
  details of a branch (parent path, sampler cursor, optimizer snapshots), so two runs that branched
  the same way from different parent files compare as matched;
* runs whose current policy agrees but whose histories differ compare as different on the history;
* a missing history is unknown, a history with a legacy first segment is partial, and neither is
  ever assumed equal to anything;
* a malformed segment, a history whose last segment disagrees with the recorded policy, one that
  goes backwards, or a branch without its rate scale or auxiliary rate, makes the history unknown.
"""
import copy

import pytest

from tensor_train_ing_b200.evaluate import _training_comparison, _training_descriptor


def _branched_run():
    """A run that trained at 16 tokens per update for 4 updates, then branched to 48 with the rate
    tripled, and has reached 160 tokens over 6 updates."""
    return {"config": {"train": {"global_prediction_tokens_per_update": 48, "lr": 0.03, "aux_adamw_lr": None}},
            "progress": {"tokens": 160, "steps": 6, "batch_history": [
                {"batch_tokens": 16, "lr": 0.01, "aux_adamw_lr": None, "start_tokens": 0, "start_step": 0,
                 "source": "fresh"},
                {"batch_tokens": 48, "lr": 0.03, "aux_adamw_lr": None, "start_tokens": 64, "start_step": 4,
                 "source": "batch_branch", "lr_scale": 3.0, "parent": {"path": "/runs/p/milestone-64"},
                 "source_sampler": {"cursor": 17}, "optimizer_groups_before": [{"lr": 0.01}],
                 "optimizer_groups_after": [{"lr": 0.03}]}]}}


def _history_status(left, right=None):
    right = left if right is None else right
    dims = _training_comparison({"training_descriptor": _training_descriptor(left)},
                                {"training_descriptor": _training_descriptor(right)})["dimensions"]
    return dims


def test_a_complete_history_keeps_the_segments_and_drops_artifact_details():
    run = _branched_run()
    untouched = copy.deepcopy(run)
    d = _training_descriptor(run)
    assert run == untouched  # the payload is only read
    assert d["batch_history_status"] == "complete"
    assert d["batch_history"] == [
        {"batch_tokens": 16, "lr": 0.01, "aux_adamw_lr": None, "start_tokens": 0, "start_step": 0,
         "source": "fresh", "lr_scale": 1.0},
        {"batch_tokens": 48, "lr": 0.03, "aux_adamw_lr": None, "start_tokens": 64, "start_step": 4,
         "source": "batch_branch", "lr_scale": 3.0}]
    elsewhere = _branched_run()
    elsewhere["progress"]["batch_history"][1].update(parent={"path": "/other/parent"}, source_sampler={"cursor": 5})
    assert _history_status(run, elsewhere)["batch_history"]["status"] == "matched"


def test_the_same_current_policy_does_not_hide_a_different_history():
    later = _branched_run()
    later["progress"]["batch_history"][1].update(start_tokens=96, start_step=6)
    later["progress"]["tokens"], later["progress"]["steps"] = 192, 8
    dims = _history_status(_branched_run(), later)
    assert dims["lr"]["status"] == dims["global_prediction_tokens_per_update"]["status"] == "matched"
    assert dims["batch_history"]["status"] == "different"


def test_missing_and_partial_histories_are_never_equal():
    missing = _branched_run()
    del missing["progress"]["batch_history"]
    assert _training_descriptor(missing)["batch_history_status"] == "unknown"
    assert _history_status(missing)["batch_history"]["status"] == "unknown"
    legacy = _branched_run()
    legacy["progress"]["batch_history"][0].update(source="legacy_unknown", start_tokens=None, start_step=None)
    d = _training_descriptor(legacy)
    assert d["batch_history_status"] == "partial" and d["batch_history"][0]["start_step"] is None
    assert _history_status(legacy)["batch_history"]["status"] == "unknown"


@pytest.mark.parametrize("segment,field,value", [
    (0, "source", "batch_branch"),      # the first segment is the fresh start
    (0, "start_step", 2),               # ... at step 0
    (0, "lr_scale", 0.5),               # ... with no rescale
    (0, "batch_tokens", 0), (0, "batch_tokens", False), (0, "lr", float("inf")), (0, "lr", -1.0),
    (1, "source", "fresh"),             # later segments are branches
    (1, "start_tokens", 161),           # past the run's tokens
    (1, "start_step", 7),               # past the run's steps
    (1, "start_step", 1.5), (1, "lr_scale", -3.0), (1, "lr_scale", float("nan")),
    (1, "batch_tokens", 32),            # the last segment disagrees with the recorded quota
    (1, "lr", 0.05),                    # ... or rate
    (1, "aux_adamw_lr", 0.01),          # ... or auxiliary rate
])
def test_malformed_or_inconsistent_segments_make_the_history_unknown(segment, field, value):
    run = _branched_run()
    run["progress"]["batch_history"][segment][field] = value
    d = _training_descriptor(run)
    assert d["batch_history"] is None and d["batch_history_status"] == "unknown"


def test_a_history_that_goes_backwards_is_unknown():
    run = _branched_run()
    back = copy.deepcopy(run["progress"]["batch_history"][1])
    back.update(start_tokens=48, start_step=3, lr_scale=1.0)
    run["progress"]["batch_history"].append(back)
    assert _training_descriptor(run)["batch_history_status"] == "unknown"


@pytest.mark.parametrize("field", ["lr_scale", "aux_adamw_lr"])
def test_a_branch_without_its_policy_evidence_is_unknown(field):
    run = _branched_run()
    del run["progress"]["batch_history"][1][field]
    assert _training_descriptor(run)["batch_history_status"] == "unknown"


def test_the_auxiliary_rate_is_its_own_evidence():
    run = _branched_run()
    run["config"]["train"]["aux_adamw_lr"] = 0.006
    run["progress"]["batch_history"][0]["aux_adamw_lr"] = 0.002
    run["progress"]["batch_history"][1]["aux_adamw_lr"] = 0.006
    assert _training_descriptor(run)["batch_history_status"] == "complete"
