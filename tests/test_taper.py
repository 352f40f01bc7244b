"""TaperNorm (``TaperRMS``) and its training lifecycle (``TaperPolicy``, ``TaperLifecycle``) on CPU:

* gate 1 is RMSNorm with the module's weight; gate 0 is the fixed diagonal map ``c * weight_tilde``,
  and a frozen all-taper model at gate 0 audits as polynomial (class "P");
* ``freeze`` sets c to the least-squares match of the linear branch to the normalised one and s_tgt
  to the mean RMS, from the bias-corrected statistics, and refuses to freeze without statistics;
* the anchor term (r - s_tgt)^2 is differentiable and resets when read;
* the gate follows a half cosine from the warm-up's end to the end step;
* the policy refuses invalid settings, the lifecycle refuses a frozen model inside its warm-up and
  updates out of order.
"""
import math

import pytest
import torch

from helpers import TINY_MODEL
from tensor_train_ing_b200.config import Config, ModelConfig, TrainConfig
from tensor_train_ing_b200.models.model import TensorLM
from tensor_train_ing_b200.models.normalization import (TaperRMS, taper_anchor_loss, taper_modules,
                                                        taper_set_gate_)
from tensor_train_ing_b200.training_taper import TaperLifecycle, TaperPolicy, taper_gate


def _rms(x, eps=1e-6):
    return (x.pow(2).mean(-1, keepdim=True) + eps).sqrt()


def _calibrated(d=16, steps=1, seed=0):
    torch.manual_seed(seed)
    norm = TaperRMS(d).double()
    with torch.no_grad():
        norm.weight.copy_(torch.rand(d, dtype=torch.float64) + 0.5)
    xs = [torch.randn(3, 5, d, dtype=torch.float64) * (1 + i) for i in range(steps)]
    norm.collecting = True
    for x in xs:
        norm(x)
        norm.commit(distributed=False)
    norm.collecting = False
    return norm, xs


def test_gate_one_is_rmsnorm_and_gate_zero_is_a_fixed_diagonal():
    norm, xs = _calibrated()
    x = xs[0]
    torch.testing.assert_close(norm(x), x / _rms(x) * norm.weight, rtol=1e-12, atol=1e-12)
    norm.freeze()
    norm.gate.fill_(0.0)
    torch.testing.assert_close(norm(x), float(norm.c) * x * norm.weight_tilde, rtol=1e-12, atol=1e-12)
    norm.gate.fill_(0.25)
    mixed = 0.25 * x / _rms(x) * norm.weight + 0.75 * float(norm.c) * x * norm.weight_tilde
    torch.testing.assert_close(norm(x), mixed, rtol=1e-12, atol=1e-12)


@pytest.mark.parametrize("steps", [1, 4])
def test_freeze_is_the_bias_corrected_least_squares_match(steps):
    norm, xs = _calibrated(steps=steps, seed=steps)
    mu = norm.ema_rate
    num = den = r_sum = 0.0
    for i, x in enumerate(xs):  # EMA over per-step token means, weight (1 - mu)^(steps - 1 - i) * mu
        w = mu * (1 - mu) ** (steps - 1 - i)
        sq = (x * norm.weight.detach()).pow(2).sum(-1)
        r = _rms(x).squeeze(-1)
        num += w * float((sq / r).mean())
        den += w * float(sq.mean())
        r_sum += w * float(r.mean())
    correction = 1 - (1 - mu) ** steps
    norm.freeze()
    assert bool(norm.frozen) and torch.equal(norm.weight_tilde.detach(), norm.weight.detach())
    assert float(norm.c) == pytest.approx((num / correction) / (den / correction), rel=1e-10)
    assert float(norm.s_tgt) == pytest.approx(r_sum / correction, rel=1e-10)


def test_freeze_needs_statistics():
    with pytest.raises(RuntimeError, match="warm-up statistic"):
        TaperRMS(8).freeze()


def test_anchor_is_differentiable_and_resets_when_read():
    norm, xs = _calibrated()
    norm.freeze()
    norm.train()
    x = xs[0].clone().requires_grad_()
    norm(x)

    class Holder(torch.nn.Module):
        def __init__(self, m):
            super().__init__()
            self.m = m
    holder = Holder(norm)
    loss = taper_anchor_loss(holder)
    want = (_rms(x).squeeze(-1) - float(norm.s_tgt)).pow(2).mean()
    torch.testing.assert_close(loss, want, rtol=1e-12, atol=1e-12)
    loss.backward()
    assert x.grad is not None and torch.isfinite(x.grad).all() and x.grad.abs().sum() > 0
    assert taper_anchor_loss(holder) is None  # read once, then reset


def test_the_gate_is_a_half_cosine_between_warmup_and_end():
    assert taper_gate(0, 10, 30) == taper_gate(10, 10, 30) == 1.0
    assert taper_gate(30, 10, 30) == taper_gate(99, 10, 30) == 0.0
    assert taper_gate(20, 10, 30) == pytest.approx(0.5)
    assert taper_gate(15, 10, 30) == pytest.approx(0.5 * (1 + math.cos(math.pi / 4)))
    values = [taper_gate(s, 10, 30) for s in range(8, 33)]
    assert all(a >= b for a, b in zip(values, values[1:]))


def _cfg(**train):
    t = dict(compile=False, bf16_compute=False)
    t.update(train)
    return Config(model=ModelConfig(**{**TINY_MODEL, "normalization": "taper", "final_normalization": "taper"}),
                  train=TrainConfig(**t), raw={})


@pytest.mark.parametrize("bad", [dict(taper_anchor_lambda=-0.1), dict(taper_end_fraction=0.0),
                                 dict(taper_end_fraction=1.5), dict(taper_anchor_lambda=float("nan")),
                                 dict(compile=True)])
def test_the_policy_refuses_invalid_settings(bad):
    with pytest.raises(ValueError):
        TaperPolicy.from_config(_cfg(**bad))


def test_the_policy_refuses_checkpointing_and_bad_ema_rates():
    cfg = _cfg()
    cfg.model.activation_checkpointing = True
    with pytest.raises(ValueError, match="checkpointing"):
        TaperPolicy.from_config(cfg)
    cfg = _cfg()
    cfg.model.taper_ema_rate = 0.0
    with pytest.raises(ValueError, match="ema_rate"):
        TaperPolicy.from_config(cfg)
    plain = Config(model=ModelConfig(**TINY_MODEL), train=TrainConfig(compile=False), raw={})
    assert TaperPolicy.from_config(plain) is None


def test_lifecycle_freezes_at_the_warmup_end_and_audits_polynomial_at_gate_zero():
    cfg = _cfg(taper_end_fraction=1.0)
    torch.manual_seed(0)
    model = TensorLM(cfg.model).double()
    life = TaperLifecycle(model, cfg, total_steps=6, warmup_steps=2)
    idx = torch.randint(0, TINY_MODEL["vocab_size"], (2, 8))
    for step in range(6):
        life.before_step(step)
        life.set_valid_mask(torch.ones(2, 8))
        loss = model(idx).float().pow(2).mean()
        anchor = life.anchor()
        if anchor is not None:
            loss = loss + anchor
        loss.backward()
        life.after_step(step + 1)
        frozen = {bool(m.frozen) for m in taper_modules(model)}
        assert frozen == ({step + 1 >= 2})
    assert all(float(m.gate) == 0.0 for m in taper_modules(model))
    assert model.operator_audit()["class"] == "P"
    taper_set_gate_(model, 0.5)
    assert model.operator_audit()["class"] == "N"
    with pytest.raises(ValueError, match="warm-up"):
        TaperLifecycle(model, cfg, total_steps=6, warmup_steps=2).before_step(1)  # frozen inside the warm-up
    life = TaperLifecycle(model, cfg, total_steps=6, warmup_steps=2)
    life.before_step(3)
    with pytest.raises(ValueError, match="exactly one"):
        life.after_step(5)
    with pytest.raises(ValueError, match="strictly after"):
        TaperLifecycle(model, cfg, total_steps=2, warmup_steps=2)
