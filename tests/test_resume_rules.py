"""The rules a parent checkpoint's recorded config must meet for a resume, a context fork or an
evaluation (runtime.resume_validator / evaluation_validator), checked on recorded configs directly:

* identical math and data resume; the token horizon may only be promoted upwards, and not at all
  under a cosine schedule or TaperNorm;
* project execution settings may change, except the spend ledger;
* a context fork needs a strictly larger context and may change nothing else;
* fields added to the schema after the checkpoint was written are accepted only at their default;
* an evaluation additionally pins the whole train section.
"""
import copy

import pytest

from tensor_train_ing_b200.config import Config, ModelConfig, TrainConfig
from tensor_train_ing_b200.runtime import evaluation_validator, full_config, resume_validator


def _cfg(**train):
    t = dict(compile=False, bf16_compute=False, lr=0.01, rung_total_tokens=1000)
    t.update(train)
    return Config(model=ModelConfig(layers=1, d_model=8, heads=1, d_key=4, d_value=4, d_mlp=12, padded_vocab=64,
                                    vocab_size=60),
                  train=TrainConfig(**t),
                  raw={"data": {"manifest": "m.json", "context": 16},
                       "project": {"dry_run": False, "spend_ledger": "ledger.json", "gpu_hourly_rate_usd": 0}})


def test_identical_config_resumes_and_horizon_promotes_upwards_only():
    saved = full_config(_cfg())
    assert resume_validator(_cfg())(copy.deepcopy(saved))["defaulted_fields"] == {}
    resume_validator(_cfg(rung_total_tokens=2000))(copy.deepcopy(saved))  # promotion
    with pytest.raises(ValueError, match="promoted upwards"):
        resume_validator(_cfg(rung_total_tokens=500))(copy.deepcopy(saved))
    with pytest.raises(ValueError, match="differs: train.lr"):
        resume_validator(_cfg(lr=0.02))(copy.deepcopy(saved))


def test_cosine_and_taper_runs_keep_their_horizon():
    saved = full_config(_cfg(schedule="cosine"))
    with pytest.raises(ValueError, match="cosine resume"):
        resume_validator(_cfg(schedule="cosine", rung_total_tokens=2000))(copy.deepcopy(saved))
    resume_validator(_cfg(schedule="cosine"))(copy.deepcopy(saved))


def test_execution_settings_may_change_but_not_the_ledger():
    saved = full_config(_cfg())
    cfg = _cfg()
    cfg.raw["project"]["dry_run"] = True
    cfg.raw["project"]["gpu_hourly_rate_usd"] = 3.5
    resume_validator(cfg)(copy.deepcopy(saved))
    cfg.raw["project"]["spend_ledger"] = "other.json"
    with pytest.raises(ValueError, match="spend ledger"):
        resume_validator(cfg)(copy.deepcopy(saved))


def test_context_fork_needs_a_larger_context_and_nothing_else():
    saved = full_config(_cfg())
    larger = _cfg()
    larger.raw["data"]["context"] = 32
    with pytest.raises(ValueError, match="differs: data.context"):
        resume_validator(larger)(copy.deepcopy(saved))  # a plain resume may not change the context
    resume_validator(larger, context_fork=True)(copy.deepcopy(saved))
    smaller = _cfg()
    smaller.raw["data"]["context"] = 8
    with pytest.raises(ValueError, match="strictly increasing"):
        resume_validator(smaller, context_fork=True)(copy.deepcopy(saved))
    larger_and_lr = _cfg(lr=0.5)
    larger_and_lr.raw["data"]["context"] = 32
    with pytest.raises(ValueError, match="train.lr"):
        resume_validator(larger_and_lr, context_fork=True)(copy.deepcopy(saved))
    with pytest.raises(ValueError):
        resume_validator(larger, context_fork="yes")


def test_fields_newer_than_the_checkpoint_must_hold_their_default():
    saved = full_config(_cfg())
    del saved["train"]["grad_clip"]  # a checkpoint written before the field existed
    record = resume_validator(_cfg())(copy.deepcopy(saved))
    assert record["defaulted_fields"] == {"train.grad_clip": TrainConfig().grad_clip}
    with pytest.raises(ValueError, match="requires its dataclass default"):
        resume_validator(_cfg(grad_clip=TrainConfig().grad_clip * 2 + 1))(copy.deepcopy(saved))


def test_evaluation_pins_the_train_section():
    saved = full_config(_cfg())
    evaluation_validator(_cfg())(copy.deepcopy(saved))
    with pytest.raises(ValueError):
        evaluation_validator(_cfg(rung_total_tokens=2000))(copy.deepcopy(saved))
