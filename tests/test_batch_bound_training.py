"""QK-clip from the training forward's own score bounds (``train.qk_clip_source: batch_bound``) in
the serial trainer, on CPU:

* with ``qk_clip_tau: 0`` the bounds are recorded (``score_bound_max`` in every metrics row) and
  nothing is clipped; the fixed-row stability probe is never built for the batch-bound source;
* the recorded maximum covers every micro-batch of the update while the clip uses the last one;
* a clipped run interrupted and resumed equals the uninterrupted run bit for bit;
* a negative or non-finite bound aborts the update before the optimizer steps;
* an unknown source is refused even when clipping is off.
"""
import copy
import json

import pytest
import torch

from helpers import state
from tensor_train_ing_b200 import training_stability
from tensor_train_ing_b200.train import train_run


def _cfg(config, tau=0.0, every=0, **train):
    cfg = copy.deepcopy(config)
    cfg.train.qk_clip_source = "batch_bound"
    cfg.train.qk_clip_tau = tau
    cfg.train.qk_clip_every_steps = every
    for k, v in train.items():
        setattr(cfg.train, k, v)
    return cfg


def _rows(path):
    return [json.loads(x) for x in (path / "metrics.jsonl").read_text().splitlines()]


@pytest.fixture
def no_probe(monkeypatch):
    def refuse(*args, **kwargs):
        raise AssertionError("the batch-bound source must not build the fixed-row probe")
    monkeypatch.setattr(training_stability.TrainingStabilityProbe, "__init__", refuse)


def test_tau_zero_records_bounds_without_clipping(config, tmp_path, no_probe):
    train_run(_cfg(config), tmp_path / "run", max_steps=2, max_seconds=120, device="cpu")
    rows = _rows(tmp_path / "run")
    assert len(rows) == 2 and all(r["score_bound_max"] > 0 and "qk_clip" not in r for r in rows)


def test_the_maximum_spans_every_micro_batch_and_the_clip_uses_the_last(config, tmp_path, monkeypatch):
    seen = []
    real_observe = training_stability.BatchScoreBounds.observe
    real_clip = training_stability.BatchScoreBounds.clip

    def observe(self):
        real_observe(self)
        seen.append([{f: b.clone() for f, b in layer.items()} for layer in self.last])

    clipped_from = []

    def clip(self, tau):
        clipped_from.append([{f: b.clone() for f, b in layer.items()} for layer in self.last])
        return real_clip(self, tau)
    monkeypatch.setattr(training_stability.BatchScoreBounds, "observe", observe)
    monkeypatch.setattr(training_stability.BatchScoreBounds, "clip", clip)
    cfg = _cfg(config, tau=1e-3, every=1)
    micro = cfg.raw["data"]["micro_batch_size"]
    cfg.train.global_prediction_tokens_per_update = 3 * micro * cfg.raw["data"]["context"]  # several micro-batches
    train_run(cfg, tmp_path / "run", max_steps=1, max_seconds=120, device="cpu")
    row = _rows(tmp_path / "run")[0]
    assert len(seen) > 1
    top = max(float(b.max()) for mb in seen for layer in mb for b in layer.values())
    assert row["score_bound_max"] == pytest.approx(top, rel=1e-6)
    assert len(clipped_from) == 1
    for layer_last, layer_clip in zip(seen[-1], clipped_from[0]):
        assert all(torch.equal(layer_last[f], layer_clip[f]) for f in layer_last)
    assert row["qk_clip"]["max_bound_before"] == pytest.approx(
        max(float(b.max()) for layer in seen[-1] for b in layer.values()), rel=1e-6)


def test_a_clipped_run_resumes_exactly(config, tmp_path, no_probe):
    cfg = _cfg(config, tau=1e-3, every=1, deterministic=True)
    train_run(cfg, tmp_path / "full", max_steps=4, max_seconds=120, device="cpu")
    first = train_run(cfg, tmp_path / "a", max_steps=2, max_seconds=120, device="cpu")
    train_run(cfg, tmp_path / "b", max_steps=2, max_seconds=120, device="cpu", resume=first["checkpoint"])
    a, b = state(tmp_path / "full" / "final"), state(tmp_path / "b" / "final")
    for k, v in a["model"].items():
        assert torch.equal(v, b["model"][k]), k
    assert [r["loss"] for r in _rows(tmp_path / "full")][2:] == [r["loss"] for r in _rows(tmp_path / "b")]
    assert _rows(tmp_path / "full")[0]["qk_clip"]["clipped_heads"] > 0


def test_a_bad_bound_aborts_before_the_optimizer_steps(config, tmp_path, monkeypatch):
    from tensor_train_ing_b200 import qk_clip
    real = qk_clip.score_bounds

    def poisoned(model):
        return [{f: torch.full_like(b, -1.0) for f, b in layer.items()} for layer in real(model)]
    monkeypatch.setattr(qk_clip, "score_bounds", poisoned)
    steps = []
    real_step = torch.optim.Optimizer.step
    monkeypatch.setattr(torch.optim.Optimizer, "step", lambda self, *a, **k: steps.append(1) or real_step(self, *a, **k))
    with pytest.raises(FloatingPointError, match="score bound"):
        train_run(_cfg(config), tmp_path / "run", max_steps=2, max_seconds=120, device="cpu")
    assert not steps
    assert not (tmp_path / "run" / "final").exists()


@pytest.mark.parametrize("source", ["batch", "probe-and-bound", ""])
def test_an_unknown_source_is_refused_even_without_clipping(config, tmp_path, source):
    cfg = _cfg(config)
    cfg.train.qk_clip_source = source
    with pytest.raises(ValueError, match="qk_clip_source"):
        train_run(cfg, tmp_path / "run", max_steps=1, max_seconds=120, device="cpu")
    assert not (tmp_path / "run").exists()
