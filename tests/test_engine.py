"""TrainEngine, the one-call optimizer update, on one CPU rank (reference path): micro-batch
invariance, the loss-normalization contract (gradient of sum(loss) / valid targets), clipping and the
learning-rate multiplier.  The multi-rank and fused-kernel paths are covered by the gloo and GPU
equivalence tests."""
import copy

import pytest
import torch

from tensor_train_ing_b200.config import Config, ModelConfig, TrainConfig
from tensor_train_ing_b200.engine import TrainEngine
from tensor_train_ing_b200.models.model import TensorLM


def _cfg(optimizer="adamw", grad_clip=0.0):
    return Config(model=ModelConfig(layers=2, d_model=16, heads=2, d_key=8, d_value=8, d_mlp=24, vocab_size=40,
                                    padded_vocab=64),
                  train=TrainConfig(optimizer=optimizer, lr=1e-2, aux_adamw_lr=1e-2, grad_clip=grad_clip,
                                    compile=False, bf16_compute=False))


def _batch(rows=4, T=10, seed=0):
    g = torch.Generator().manual_seed(seed)
    toks = torch.randint(0, 40, (rows, T + 1), generator=g)
    docs = torch.zeros(rows, T, dtype=torch.long)
    docs[1, 6:] = 1  # a second document in one row
    targets = toks[:, 1:].clone()
    targets[1, 5] = -100  # no target across the document boundary
    targets[3] = -100     # a row with nothing scored
    return toks[:, :T], docs, targets


def _engine(cfg, micro_batch, seed=0):
    torch.manual_seed(seed)
    model = TensorLM(cfg.model)
    return TrainEngine(cfg, device="cpu", micro_batch=micro_batch, model=model)


@pytest.mark.parametrize("optimizer", ["adamw", "muon"])
def test_micro_batch_split_does_not_change_the_update(optimizer):
    torch.set_num_threads(1)
    cfg = _cfg(optimizer)
    a, b = _engine(cfg, 4), _engine(cfg, 1)
    batch = _batch()
    for step in range(2):
        la, ca = a.step(*batch)
        lb, cb = b.step(*batch)
        assert int(ca) == int(cb) == int((batch[2] != -100).sum())
        torch.testing.assert_close(la, lb, rtol=1e-5, atol=1e-6)
    # Muon's Newton-Schulz iterations run in reduced precision and amplify rounding-level gradient
    # differences (about 1e-4 on weights of order 1 after two steps); AdamW stays at rounding level
    atol = 5e-4 if optimizer == "muon" else 1e-6
    for (k, pa), pb in zip(a.model.named_parameters(), b.model.parameters()):
        torch.testing.assert_close(pa, pb, rtol=1e-4, atol=atol, msg=lambda m, k=k: f"{k}: {m}")


def test_gradients_follow_the_loss_normalization_contract():
    torch.set_num_threads(1)
    cfg = _cfg()
    eng = _engine(cfg, 2)
    ref = copy.deepcopy(eng.model)
    idx, docs, targets = _batch()
    loss_sum, count = eng.step(idx, docs, targets)
    _, loss, n = ref(idx, docs, targets, reduction="sum")
    torch.testing.assert_close(loss_sum, loss.detach(), rtol=1e-5, atol=1e-6)
    (loss / n).backward()
    for (k, p), q in zip(eng.model.named_parameters(), ref.parameters()):
        assert p.grad is not None, k
        torch.testing.assert_close(p.grad, q.grad, rtol=1e-4, atol=1e-7, msg=lambda m, k=k: f"{k}: {m}")


def test_clipping_bounds_the_global_norm_and_lr_multiplier_scales_from_base():
    torch.set_num_threads(1)
    eng = _engine(_cfg(grad_clip=1e-3), 4)
    eng.step(*_batch())
    assert float(eng.last_grad_norm) > 1e-3  # the pre-clip norm is reported
    clipped = torch.sqrt(sum((p.grad.double() ** 2).sum() for p in eng.model.parameters() if p.grad is not None))
    assert float(clipped) == pytest.approx(1e-3, rel=1e-3)
    base = [g.get("base_lr", g["lr"]) for g in eng.optimizer.param_groups]
    eng.step(*_batch(seed=1), lr_multiplier=0.25)
    assert [g["lr"] for g in eng.optimizer.param_groups] == pytest.approx([0.25 * b for b in base])


@pytest.mark.parametrize("recompute", [None, 0, 1, 2])
def test_selective_recompute_keeps_every_gradient(recompute, monkeypatch):
    """Under activation checkpointing, recomputing only the first ``recompute`` blocks (keeping the
    other blocks' activations) gives bit-identical gradients to recomputing all of them; the model
    reports how many it recomputes."""
    cfg = _cfg()
    cfg.model.activation_checkpointing = True
    monkeypatch.delenv("TTB_RECOMPUTE_BLOCKS", raising=False)
    torch.manual_seed(0)
    ref = TrainEngine(cfg, device="cpu", micro_batch=2, model=TensorLM(cfg.model))
    torch.manual_seed(0)
    eng = TrainEngine(cfg, device="cpu", micro_batch=2, model=TensorLM(cfg.model), recompute_blocks=recompute)
    assert eng.model.recomputed_blocks() == (2 if recompute is None else recompute)
    idx, docs, tgt = _batch()
    for e in (ref, eng):
        e.begin_update()
        inv = torch.tensor(1.0 / float((tgt != -100).sum()))
        e.forward_backward(idx, docs, tgt, inv)
    for (name, a), b in zip(ref.model.named_parameters(), eng.model.parameters()):
        assert (a.grad is None) == (b.grad is None), name
        if a.grad is not None:
            assert torch.equal(a.grad, b.grad), name
    eng.model.eval()
    assert eng.model.recomputed_blocks() == 0  # evaluation keeps nothing to recompute


def test_recompute_blocks_from_the_environment(monkeypatch):
    cfg = _cfg()
    cfg.model.activation_checkpointing = True
    monkeypatch.setenv("TTB_RECOMPUTE_BLOCKS", "1")
    eng = _engine(cfg, 2)
    assert eng.model.recomputed_blocks() == 1
