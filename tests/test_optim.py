"""Optimizer rules: parameter split, Muon == torch.optim.Muon, AdamW decay groups, LR scaling."""
import pytest
import torch

from helpers import TINY_MODEL
from tensor_train_ing_b200.config import ModelConfig, TrainConfig
from tensor_train_ing_b200.models.model import TensorLM
from tensor_train_ing_b200.optim import Muon, MuonAdamW, make_optimizer, newton_schulz, param_split


def _model(**kw):
    torch.manual_seed(0)
    return TensorLM(ModelConfig(**{**TINY_MODEL, **kw}))


def test_split_keeps_logical_matrices_separate():
    m = _model()
    hidden, vocab, small = param_split(m)
    names = {id(p): n for n, p in m.named_parameters()}
    assert all(p.dim() == 2 for p in hidden)
    assert {names[id(p)] for p in vocab} == {"embed.weight", "unembed.weight"}
    assert all(p.dim() < 2 for p in small)
    assert len(hidden) + len(vocab) + len(small) == len(list(m.parameters()))


@pytest.mark.skipif(not hasattr(torch.optim, "Muon"), reason="torch.optim.Muon not available")
@pytest.mark.parametrize("rule", ["original", "match_rms_adamw"])
def test_muon_matches_torch_muon(rule):
    torch.manual_seed(1)
    w0 = torch.randn(16, 24)
    grads = [torch.randn(16, 24) for _ in range(3)]
    a = torch.nn.Parameter(w0.clone())
    b = torch.nn.Parameter(w0.clone())
    ours = Muon([a], lr=0.02, weight_decay=0.1, momentum=0.9, adjust_lr_fn=rule)
    ref = torch.optim.Muon([b], lr=0.02, weight_decay=0.1, momentum=0.9, adjust_lr_fn=rule)
    for g in grads:
        a.grad, b.grad = g.clone(), g.clone()
        ours.step()
        ref.step()
    torch.testing.assert_close(a.detach(), b.detach(), rtol=1e-5, atol=1e-5)


def test_newton_schulz_orthogonalizes():
    torch.manual_seed(2)
    g = torch.randn(32, 64)
    o = newton_schulz(g).float()
    s = torch.linalg.svdvals(o)
    assert s.max() < 1.3 and s.min() > 0.5


def test_muon_trains_and_state_roundtrips():
    m = _model()
    opt = make_optimizer(m, TrainConfig(optimizer="muon", lr=0.01))
    assert isinstance(opt, MuonAdamW)
    idx = torch.randint(0, 97, (4, 8))
    losses = []
    for _ in range(5):
        opt.zero_grad()
        _, loss = m(idx, targets=torch.roll(idx, -1, 1))
        loss.backward()
        opt.step()
        losses.append(float(loss))
    assert losses[-1] < losses[0]
    sd = opt.state_dict()
    assert set(sd) == {"muon", "adamw"}
    opt2 = make_optimizer(m, TrainConfig(optimizer="muon", lr=0.01))
    opt2.load_state_dict(sd)
    assert len(opt2.state) == len(opt.state)


def test_adamw_groups_decay_only_hidden_matrices():
    m = _model()
    opt = make_optimizer(m, TrainConfig(optimizer="adamw", lr=0.01, weight_decay_hidden=0.1))
    hidden, vocab, small = param_split(m)
    decayed = {id(p) for g in opt.param_groups if g["weight_decay"] > 0 for p in g["params"]}
    assert decayed == {id(p) for p in hidden}


def test_width_scaling_lr_and_logit_multiplier():
    m = _model(width_scaling_base=16)
    opt = make_optimizer(m, TrainConfig(optimizer="adamw", lr=0.01))
    hidden_group = next(g for g in opt.param_groups if g["weight_decay"] > 0)
    assert hidden_group["lr"] == pytest.approx(0.01 * (16 / 32) ** 0.5)
    assert m.logit_multiplier == pytest.approx((16 / 32) ** 0.5)
