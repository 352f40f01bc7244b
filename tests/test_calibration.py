"""Lagged-norm calibration through its collective-control path, driven by stub collectives in one
process (no process group): the statistics equal the serial path's, every agreement point is
reached in order, and a failed agreement leaves all statistics and module modes as they were
(the reference checks the same path with mocked `_phase`/`_agree`,
tests/test_distributed_calibration.py)."""
import time

import pytest
import torch

from tensor_train_ing_b200 import distributed_checkpoint as dc
from tensor_train_ing_b200.calibration import calibrate_lagged
from tensor_train_ing_b200.config import Config, ModelConfig
from tensor_train_ing_b200.models.model import TensorLM
from tensor_train_ing_b200.models.normalization import lagged_modules


def _lagged(config):
    model = ModelConfig(layers=2, d_model=8, heads=1, d_key=4, d_value=4, d_mlp=12, padded_vocab=50257,
                        normalization="lagged", final_normalization="lagged")
    return Config(model=model, train=config.train, raw=config.raw)


def _stats(model):
    return {n: {k: v.clone() for k, v in m.named_buffers()} for n, m in model.named_modules() if m in
            set(lagged_modules(model))}


def _stub_collectives(monkeypatch, log, fail_at=None):
    monkeypatch.setattr(torch.distributed, "is_initialized", lambda: True)
    monkeypatch.setattr(torch.distributed, "get_world_size", lambda group=None: 1)

    def phase(label, fn):
        log.append(("phase", label))
        return fn()

    def agree(label, value):
        log.append(("agree", label))
        if label == fail_at:
            raise RuntimeError(f"ranks disagree at {label}")
    monkeypatch.setattr(dc, "_phase", phase)
    monkeypatch.setattr(dc, "_agree", agree)


def test_collective_control_with_one_rank_matches_the_serial_calibration(config, monkeypatch):
    cfg = _lagged(config)
    manifest = cfg.raw["data"]["manifest"]
    torch.manual_seed(0)
    serial = TensorLM(cfg.model)
    torch.manual_seed(0)
    collective = TensorLM(cfg.model)
    r1 = calibrate_lagged(serial, cfg, manifest, "cpu", deadline=time.monotonic() + 120)
    log = []
    _stub_collectives(monkeypatch, log)
    r2 = calibrate_lagged(collective, cfg, manifest, "cpu", deadline=time.monotonic() + 120, collective_control=True)
    assert r1 == r2 and r1["tokens"] > 0 and r1["passes"] == len(lagged_modules(serial))
    s1, s2 = _stats(serial), _stats(collective)
    assert s1.keys() == s2.keys() and s1
    for name in s1:
        for k in s1[name]:
            assert torch.equal(s1[name][k], s2[name][k]), (name, k)
    agreements = [label for kind, label in log if kind == "agree"]
    assert agreements[0] == "calibration prefix/site identity"
    assert agreements[-1] == "calibration complete report"
    assert agreements.count("calibration committed site") == r2["passes"]
    assert ("phase", "calibration setup") in log


def test_a_failed_agreement_restores_statistics_and_modes(config, monkeypatch):
    cfg = _lagged(config)
    torch.manual_seed(0)
    model = TensorLM(cfg.model)
    model.train()
    before = _stats(model)
    _stub_collectives(monkeypatch, [], fail_at="calibration committed site")
    with pytest.raises(RuntimeError, match="disagree"):
        calibrate_lagged(model, cfg, cfg.raw["data"]["manifest"], "cpu", deadline=time.monotonic() + 120,
                         collective_control=True)
    assert all(m.training for m in model.modules())
    after = _stats(model)
    for name in before:
        for k in before[name]:
            assert torch.equal(before[name][k], after[name][k]), (name, k)
    assert not any(m.collecting for m in lagged_modules(model))


def test_collective_control_needs_a_process_group_and_replicated_statistics(config, monkeypatch):
    cfg = _lagged(config)
    model = TensorLM(cfg.model)
    with pytest.raises(ValueError, match="process group"):
        calibrate_lagged(model, cfg, cfg.raw["data"]["manifest"], "cpu", deadline=time.monotonic() + 60,
                         collective_control=True)
    _stub_collectives(monkeypatch, [])
    with pytest.raises(ValueError, match="distributed=False"):
        calibrate_lagged(model, cfg, cfg.raw["data"]["manifest"], "cpu", deadline=time.monotonic() + 60,
                         collective_control=True, distributed=True)
