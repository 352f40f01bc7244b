"""Periodic stability logging (``train.stability_every_steps``) in the serial trainer, on CPU:

* the probe runs on a fixed row at its cadence and leaves training untouched: losses, weights and the
  RNG stream equal a run without it, and a probed run resumes exactly;
* with the cadence 0 (the default) no probe is built;
* malformed cadences are refused before the run writes anything.
"""
import copy
import json

import pytest
import torch

from helpers import state
from tensor_train_ing_b200 import training_stability
from tensor_train_ing_b200.train import train_run


def _rows(path):
    return [json.loads(x) for x in (path / "metrics.jsonl").read_text().splitlines()]


def _cfg(config, every):
    cfg = copy.deepcopy(config)
    cfg.train.stability_every_steps = every
    cfg.train.deterministic = True
    return cfg


def test_the_probe_leaves_training_untouched_and_resumes(config, tmp_path):
    plain = train_run(_cfg(config, 0), tmp_path / "plain", max_steps=4, max_seconds=120, device="cpu")
    probed = train_run(_cfg(config, 2), tmp_path / "probed", max_steps=4, max_seconds=120, device="cpu")
    rows = _rows(tmp_path / "probed")
    assert [("stability" in r) for r in rows] == [False, True, False, True]
    assert [r["loss"] for r in rows] == [r["loss"] for r in _rows(tmp_path / "plain")]
    a, b = state(tmp_path / "plain" / "final"), state(tmp_path / "probed" / "final")
    for k, v in a["model"].items():
        assert torch.equal(v, b["model"][k]), k
    assert probed["progress"]["tokens"] == plain["progress"]["tokens"]
    first = train_run(_cfg(config, 2), tmp_path / "a", max_steps=3, max_seconds=120, device="cpu")
    train_run(_cfg(config, 2), tmp_path / "b", max_steps=1, max_seconds=120, device="cpu",
              resume=first["checkpoint"])
    c = state(tmp_path / "b" / "final")
    for k, v in b["model"].items():
        assert torch.equal(v, c["model"][k]), k
    resumed_rows = _rows(tmp_path / "b")
    assert resumed_rows[0]["step"] == 4 and "stability" in resumed_rows[0]
    strip = lambda report: {k: v for k, v in report.items() if k != "seconds"}  # noqa: E731
    assert strip(resumed_rows[0]["stability"]) == strip(rows[3]["stability"])


def test_no_probe_is_built_when_the_cadence_is_zero(config, tmp_path, monkeypatch):
    def refuse(*args, **kwargs):
        raise AssertionError("a probe was built with periodic logging off")
    monkeypatch.setattr(training_stability.TrainingStabilityProbe, "__init__", refuse)
    train_run(_cfg(config, 0), tmp_path / "run", max_steps=1, max_seconds=120, device="cpu")
    assert all("stability" not in r for r in _rows(tmp_path / "run"))


@pytest.mark.parametrize("every", [-1, True, 1.5, "2"])
def test_a_malformed_cadence_is_refused_before_any_write(config, tmp_path, every):
    with pytest.raises(ValueError, match="stability_every_steps"):
        train_run(_cfg(config, every), tmp_path / "run", max_steps=1, max_seconds=120, device="cpu")
    assert not (tmp_path / "run").exists()
