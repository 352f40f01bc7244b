"""QK-clip (probe and per-batch bounds), the per-update score-bound tracker and the TaperNorm
lifecycle (CPU, fp64)."""
import types

import pytest
import torch

from helpers import TINY_MODEL
from tensor_train_ing_b200.config import Config, ModelConfig, TrainConfig
from tensor_train_ing_b200.models.model import TensorLM
from tensor_train_ing_b200.qk_clip import head_score_max, qk_clip_, qk_clip_from_bounds_, score_bounds, \
    set_score_bound_recording
from tensor_train_ing_b200.training_stability import BatchScoreBounds, StabilityPolicy
from tensor_train_ing_b200.training_taper import TaperLifecycle, validate_taper_config


@pytest.fixture
def fp64():
    old = torch.get_default_dtype()
    torch.set_default_dtype(torch.float64)
    yield
    torch.set_default_dtype(old)


def _model(**kw):
    torch.manual_seed(0)
    cfg = ModelConfig(**{**TINY_MODEL, "qk_init_scale": 4.0, **kw})
    return TensorLM(cfg)


def _batch(T=24):
    g = torch.Generator().manual_seed(3)
    idx = torch.randint(0, 97, (2, T), generator=g)
    doc = torch.zeros(2, T, dtype=torch.long)
    doc[:, T // 2:] = 1
    return idx, doc


def test_probe_qk_clip_caps_every_head_at_tau(fp64):
    model = _model()
    idx, doc = _batch()
    before = head_score_max(model, idx, doc)
    worst = max(float(v.max()) for row in before for v in row.values())
    tau = 0.5 * worst
    report = qk_clip_(model, idx, doc, tau)
    assert report["clipped_heads"] > 0 and report["max_before"] == pytest.approx(worst)
    after = head_score_max(model, idx, doc)
    for row_b, row_a in zip(before, after):
        for name in row_b:
            # clipped heads land on tau, the others keep their value (layer 0 is exact; later layers
            # were re-measured after the earlier ones changed)
            assert float(row_a[name].max()) <= tau * (1 + 1e-9)
    assert float(after[0]["S1"].max()) == pytest.approx(tau)


def test_batch_bounds_dominate_the_true_scores_and_clip_below_tau(fp64):
    model = _model()
    idx, doc = _batch()
    true = head_score_max(model, idx, doc)  # (its probe forward would overwrite recorded bounds)
    set_score_bound_recording(model, True)
    model(idx, doc)
    bounds = score_bounds(model)
    for b_row, t_row in zip(bounds, true):
        for name, b in b_row.items():
            assert (b >= t_row[name] * (1 - 1e-12)).all()  # Cauchy-Schwarz: a bound, never below
    tau = 0.25 * max(float(b.max()) for row in bounds for b in row.values())
    report = qk_clip_from_bounds_(model, tau)
    assert report["clipped_heads"] > 0
    for i, row in report["factors"].items():  # each clipped head was scaled by tau / bound
        for name, gam in row.items():
            want = torch.clamp(tau / bounds[i][name].double(), max=1.0)
            assert torch.allclose(torch.tensor(gam, dtype=torch.float64), want, rtol=1e-6)
    model(idx, doc)
    # the first layer sees the same input, so its bounds now sit at tau; later layers' inputs moved
    for b in score_bounds(model)[0].values():
        assert float(b.max()) <= tau * (1 + 1e-5)


def test_score_bound_tracker_lifecycle(fp64):
    model = _model()
    idx, doc = _batch()
    cfg = types.SimpleNamespace(train=types.SimpleNamespace(qk_clip_source="batch_bound", qk_clip_tau=1.0,
                                                            qk_clip_every_steps=2),
                                model=types.SimpleNamespace(attention="signed_product", normalization="pre_rms"))
    policy = StabilityPolicy.from_config(cfg)
    assert (policy.clip_source, policy.clip_tau, policy.clip_every, policy.stability_every) == ("batch_bound", 1.0, 2, 0)
    tracker = BatchScoreBounds(model, cfg)
    tracker.begin_update()
    with pytest.raises(ValueError):
        tracker.finish_update()  # nothing observed
    for T in (16, 24):
        model(*_batch(T))
        tracker.observe()
    mx = tracker.finish_update()
    assert mx > 0 and len(tracker.last) == model.cfg.layers
    stats = tracker.clip(0.5 * mx)
    assert stats["clipped_heads"] > 0 and "seconds" in stats
    bad = types.SimpleNamespace(train=types.SimpleNamespace(qk_clip_source="batch_bound", qk_clip_tau=1.0,
                                                            qk_clip_every_steps=0), model=cfg.model)
    with pytest.raises(ValueError):
        StabilityPolicy.from_config(bad)  # clipping enabled with no interval


def test_taper_lifecycle_warmup_freeze_and_gate():
    mcfg = ModelConfig(**{**TINY_MODEL, "normalization": "taper", "final_normalization": "taper"})
    cfg = Config(model=mcfg, train=TrainConfig(compile=False, taper_end_fraction=0.5, taper_anchor_lambda=0.1))
    assert validate_taper_config(cfg)
    torch.manual_seed(0)
    model = TensorLM(mcfg)
    taper = TaperLifecycle(model, cfg, total_steps=40, warmup_steps=4)
    assert taper.enabled and taper.norms and taper.end_step == 20
    idx, doc = _batch()
    gates = []
    for step in range(24):
        taper.before_step(step)
        if taper.collecting:
            taper.set_valid_mask(doc >= 0)
        _, loss = model(idx, doc, torch.roll(idx, -1, 1))
        anchor = taper.anchor()
        if anchor is not None:
            assert torch.isfinite(anchor)
        taper.set_valid_mask(None)
        taper.after_step(step + 1)
        gates.append(taper.metrics(0.0).get("taper_gate"))
    known = [g for g in gates if g is not None]
    assert known and known[0] >= known[-1]  # the gate only falls
    assert known[-1] == pytest.approx(0.0, abs=1e-12)  # closed at the end fraction
    bad = Config(model=mcfg, train=TrainConfig(compile=False, taper_end_fraction=1.5))
    with pytest.raises(ValueError):
        validate_taper_config(bad)


def test_reduce_last_takes_the_per_head_maximum_over_ranks(fp64):
    """The distributed clip's agreement step: each (layer, factor, head) bound becomes the maximum of
    the ranks' values, and a rank that ran no micro-batch contributes zeros.  The reducer here plays
    two other ranks."""
    model = _model()
    cfg = Config(model=model.cfg, train=TrainConfig(qk_clip_source="batch_bound"), raw={})
    bounds = BatchScoreBounds(model, cfg)
    idx, doc = _batch()
    bounds.begin_update()
    model(idx, doc_ids=doc)
    bounds.observe()
    mine = torch.cat([b.double() for layer in bounds.last for b in layer.values()])
    other = torch.rand_like(mine) * 2 * float(mine.max())

    def reducer(flat):  # ranks: this one, one with other values, one with no micro-batch (zeros)
        flat.copy_(torch.maximum(torch.maximum(flat, other), torch.zeros_like(flat)))
    bounds.reduce_last(reducer)
    got = torch.cat([b for layer in bounds.last for b in layer.values()])
    assert torch.equal(got, torch.maximum(mine, other))
    idle = BatchScoreBounds(model, cfg)  # a rank without a micro-batch this update
    idle.begin_update()
    seen = []
    idle.reduce_last(lambda flat: seen.append(flat.clone()) or flat.copy_(torch.maximum(flat, other)))
    assert torch.equal(seen[0], torch.zeros_like(other))
    assert torch.equal(torch.cat([b for layer in idle.last for b in layer.values()]), other)
