"""Schedules, checkpoint planning / disk admission, optimizer exposure bookkeeping and the throughput
canary (CPU)."""
import errno
import json
import math
from collections import namedtuple

import pytest
import torch

from helpers import TINY_MODEL
from tensor_train_ing_b200 import checkpoint_storage
from tensor_train_ing_b200.checkpoint_plan import (checkpoint_retention_policy, checkpoint_storage_plan,
                                                   milestone_policy, pending_milestone_tokens)
from tensor_train_ing_b200.checkpoint_storage import (RESERVE_BYTES, checkpoint_space_estimate,
                                                      require_checkpoint_space)
from tensor_train_ing_b200.config import Config, ModelConfig, TrainConfig
from tensor_train_ing_b200.models.model import TensorLM
from tensor_train_ing_b200.optim import make_optimizer
from tensor_train_ing_b200.optimizer_exposure import update_optimizer_exposure
from tensor_train_ing_b200.schedules import (COSINE, CONSTANT, lr_multiplier, schedule_multiplier, schedule_steps,
                                             validate_schedule)
from tensor_train_ing_b200.throughput_canary import ThroughputCanary


# ------------------------------------------------------------------------------------- schedules
def test_warmup_is_max_of_100_and_one_percent():
    assert validate_schedule(CONSTANT, 50) == 100
    assert validate_schedule(CONSTANT, 10_000) == 100
    assert validate_schedule(CONSTANT, 10_001) == 101
    assert validate_schedule(COSINE, 30_000) == 300
    assert schedule_steps(1000, 7) == 143


def test_constant_schedule_ramps_then_holds():
    total = 1000
    assert schedule_multiplier(0, total) == pytest.approx(1 / 100)
    assert schedule_multiplier(49, total) == pytest.approx(0.5)
    assert schedule_multiplier(99, total) == 1.0
    assert schedule_multiplier(999, total) == 1.0
    assert lr_multiplier(99, total) == 1.0  # the same warm-up rule without a cooldown


def test_cosine_reaches_zero_at_the_last_update_and_is_monotone_after_warmup():
    total = 400
    vals = [schedule_multiplier(s, total, schedule=COSINE) for s in range(total)]
    assert vals[99] == 1.0 and vals[-1] == 0.0
    assert all(a >= b for a, b in zip(vals[100:], vals[101:]))
    mid = 100 + (total - 100) // 2 - 1
    assert vals[mid] == pytest.approx(0.5 * (1 + math.cos(math.pi * (mid + 1 - 100) / 300)))
    with pytest.raises(ValueError):
        schedule_multiplier(total, total, schedule=COSINE)
    with pytest.raises(ValueError):
        validate_schedule(COSINE, 100)  # no room after warm-up
    with pytest.raises(ValueError):
        validate_schedule(COSINE, 400, cooldown_steps=10)


def test_cooldown_decays_linearly_to_zero():
    assert lr_multiplier(0, 1000, cooldown_steps=10) == 1.0
    assert lr_multiplier(5, 1000, cooldown_steps=10) == 0.5
    assert lr_multiplier(10, 1000, cooldown_steps=10) == 0.0
    assert lr_multiplier(20, 1000, cooldown_steps=10) == 0.0
    with pytest.raises(ValueError):
        lr_multiplier(0, 1000, cooldown_steps=0)


@pytest.mark.parametrize("bad", [0, -1, 1.5, True])
def test_schedule_rejects_non_positive_integer_horizons(bad):
    with pytest.raises(ValueError):
        schedule_steps(bad, 7)


# ------------------------------------------------------------------------ checkpoint planning
def _cfg(project=None, **train):
    return Config(model=ModelConfig(**TINY_MODEL),
                  train=TrainConfig(global_prediction_tokens_per_update=1_000_000, rung_total_tokens=250_000_000,
                                    **train),
                  raw={"project": project or {}})


def test_default_milestones_double_then_every_100m():
    got = list(pending_milestone_tokens(_cfg(), start_tokens=0, token_limit=250_000_000))
    assert got == [1_000_000, 2_000_000, 4_000_000, 8_000_000, 16_000_000, 32_000_000, 100_000_000, 200_000_000]
    resumed = list(pending_milestone_tokens(_cfg(), start_tokens=8_000_000, token_limit=150_000_000))
    assert resumed == [16_000_000, 32_000_000, 100_000_000]
    branch = list(pending_milestone_tokens(_cfg(), start_tokens=0, token_limit=250_000_000, include_branch=True))
    assert 225_000_000 in branch and branch == sorted(set(branch))


def test_explicit_milestones_and_retention_policy_validation():
    cfg = _cfg({"milestone_tokens": [5, 3, 3, 9], "keep_recovery_checkpoints": 4, "save_initial_checkpoint": False})
    assert milestone_policy(cfg) == {"mode": "explicit", "tokens": [3, 5, 9]}
    assert list(pending_milestone_tokens(cfg, start_tokens=3, token_limit=100)) == [5, 9]
    assert checkpoint_retention_policy(cfg) == {"keep_recovery_checkpoints": 4, "save_initial_checkpoint": False}
    with pytest.raises(ValueError):
        milestone_policy(_cfg({"milestone_tokens": [0]}))
    with pytest.raises(ValueError):
        checkpoint_retention_policy(_cfg({"save_initial_checkpoint": "yes"}))


def test_storage_plan_counts_parameters_moments_and_checkpoints():
    cfg = _cfg(optimizer="adamw")
    plan = checkpoint_storage_plan(cfg)
    model = TensorLM(cfg.model)
    params = sum(p.numel() * p.element_size() for p in model.parameters())
    br = plan["tensor_bytes_breakdown"]
    assert br["parameters"] == params
    assert br["optimizer_moments"] == 2 * params  # AdamW: two fp32 moments per parameter
    assert plan["checkpoint_count"] == sum(plan["count_breakdown"].values())
    assert plan["required_additional_bytes"] >= plan["per_checkpoint_estimate_bytes"] * plan["checkpoint_count"]
    muon = checkpoint_storage_plan(_cfg(optimizer="muon"))
    assert muon["tensor_bytes_breakdown"]["optimizer_moments"] < br["optimizer_moments"]  # one moment on matrices
    dist_plan = checkpoint_storage_plan(cfg, distributed=True, distributed_world_size=4)
    assert dist_plan["tensor_bytes_breakdown"]["distributed_shard_padding_allowance"] > 0
    with pytest.raises(ValueError):
        checkpoint_storage_plan(cfg, distributed_world_size=2)  # serial plan with a world size


def test_storage_plan_builds_nothing_real_and_draws_no_random_numbers(monkeypatch):
    """The plan sizes a model built on the meta device: no parameter memory, and the Python, NumPy
    and torch generators are where they were (a plan before a run does not shift its initialisation)."""
    import random

    import numpy as np
    built = []
    original = TensorLM.__init__

    def recording(self, *args, **kwargs):
        original(self, *args, **kwargs)
        built.append({p.device.type for p in self.parameters()})
    monkeypatch.setattr(TensorLM, "__init__", recording)
    py, npy, th = random.getstate(), np.random.get_state()[1].copy(), torch.get_rng_state().clone()
    checkpoint_storage_plan(_cfg(optimizer="adamw"))
    assert built and all(kinds == {"meta"} for kinds in built)
    assert random.getstate() == py and (np.random.get_state()[1] == npy).all()
    assert torch.equal(torch.get_rng_state(), th)


def test_storage_plan_follows_the_default_dtype_and_huge_horizons_stay_json():
    base = checkpoint_storage_plan(_cfg(optimizer="adamw"), max_steps=0)
    old = torch.get_default_dtype()
    try:
        torch.set_default_dtype(torch.float64)
        double = checkpoint_storage_plan(_cfg(optimizer="adamw"), max_steps=0)
    finally:
        torch.set_default_dtype(old)
    assert double["tensor_bytes_breakdown"]["parameters"] == 2 * base["tensor_bytes_breakdown"]["parameters"]
    assert double["dtype"] == "torch.float64"
    huge = checkpoint_storage_plan(_cfg(optimizer="adamw"), token_limit=10 ** 40)
    assert huge["count_breakdown"]["milestones"] > 10 ** 30  # counted in closed form, not enumerated
    json.dumps(huge, allow_nan=False)
    exported = checkpoint_storage_plan(_cfg(optimizer="adamw"), max_steps=0, export_weights=True)
    assert exported["required_additional_bytes"] == (base["required_additional_bytes"]
                                                     + exported["export_weights_estimate_bytes"])


@pytest.mark.parametrize("bad", [{"start_tokens": -1}, {"token_limit": float("inf")}, {"max_steps": True},
                                 {"max_steps": 2.5}, {"distributed_world_size": 0}, {"cooldown": 1},
                                 {"distributed": "yes"}])
def test_storage_plan_rejects_malformed_arguments(bad):
    with pytest.raises(ValueError):
        checkpoint_storage_plan(_cfg(optimizer="adamw"), **bad)


def test_space_estimate_counts_shared_storage_once():
    a = torch.zeros(1000)
    once = checkpoint_space_estimate({"x": a})
    twice = checkpoint_space_estimate({"x": a, "view": a[10:20], "alias": a})
    assert twice - once < 1000  # only pickle metadata grows
    bigger = checkpoint_space_estimate({"x": a, "y": torch.zeros(1000)})
    assert bigger - once >= 4000
    with pytest.raises(ValueError):
        checkpoint_space_estimate({"m": torch.empty(3, device="meta")})


def test_disk_admission_keeps_a_reserve(tmp_path, monkeypatch):
    usage = namedtuple("usage", "total used free")
    monkeypatch.setattr(checkpoint_storage.shutil, "disk_usage", lambda p: usage(10 ** 12, 0, RESERVE_BYTES + 100))
    info = require_checkpoint_space(tmp_path / "not" / "yet" / "there", 100)
    assert info["free_bytes"] == RESERVE_BYTES + 100
    with pytest.raises(OSError) as exc:
        require_checkpoint_space(tmp_path, 101)
    assert exc.value.errno == errno.ENOSPC
    with pytest.raises(ValueError):
        require_checkpoint_space(tmp_path, -1)


# ------------------------------------------------------------------------- optimizer exposure
def test_exposure_accumulates_lr_and_decay_shrinkage():
    torch.manual_seed(0)
    model = TensorLM(ModelConfig(**TINY_MODEL))
    opt = make_optimizer(model, TrainConfig(optimizer="adamw", lr=0.01, weight_decay_hidden=0.1))
    progress = {"steps": 0, "tokens": 0}
    for step in range(3):
        for g in opt.param_groups:
            g["lr"] = 0.01 * (step + 1)
        update_optimizer_exposure(progress, opt)
        progress["steps"] += 1
    exp = progress["optimizer_exposure"]
    assert exp["observed_steps"] == 3 and exp["complete_history"]
    hidden = exp["groups"][0]
    assert hidden["sum_lr"] == pytest.approx(0.06)
    assert hidden["sum_lr_weight_decay"] == pytest.approx(0.006)
    want = sum(math.log1p(-0.01 * k * 0.1) for k in (1, 2, 3))
    assert hidden["shrinkage_log_abs"] == pytest.approx(want)
    json.dumps(exp, allow_nan=False)
    progress["steps"] += 5  # a gap in the observed history is refused
    with pytest.raises(ValueError):
        update_optimizer_exposure(progress, opt)


def _exposure_opt(lr=0.01, wd=0.1):
    torch.manual_seed(0)
    model = TensorLM(ModelConfig(**TINY_MODEL))
    return make_optimizer(model, TrainConfig(optimizer="adamw", lr=lr, weight_decay_hidden=wd))


def test_exposure_zero_and_negative_decay_factors_stay_finite():
    """lr * wd = 1 zeroes the shrinkage (its sign becomes 0 and the log is undefined, recorded as
    None); lr * wd > 1 flips its sign once per such update; the record stays finite JSON; a zero
    rate still counts as an update."""
    opt = _exposure_opt()
    progress = {"steps": 0, "tokens": 0}
    hidden = lambda: progress["optimizer_exposure"]["groups"][0]  # noqa: E731
    for lr, wd in ((0.0, 0.1), (3.0, 1.0), (4.0, 1.0)):
        for g in opt.param_groups:
            g["lr"] = lr
            g["weight_decay"] = wd if g["weight_decay"] else 0.0
        update_optimizer_exposure(progress, opt)
        progress["steps"] += 1
    row = hidden()
    assert row["observed_steps"] == 3 and row["sum_lr"] == pytest.approx(7.0)
    assert row["negative_factors"] == 2 and row["zero_factors"] == 0 and row["shrinkage_sign"] == 1
    assert row["shrinkage_log_abs"] == pytest.approx(math.log(2.0) + math.log(3.0))
    for g in opt.param_groups:
        g["lr"] = 1.0
        g["weight_decay"] = 1.0 if g["weight_decay"] else 0.0
    update_optimizer_exposure(progress, opt)
    assert hidden()["zero_factors"] == 1 and hidden()["shrinkage_sign"] == 0 and hidden()["shrinkage_log_abs"] is None
    json.dumps(progress["optimizer_exposure"], allow_nan=False)


def test_exposure_refuses_bad_input_without_touching_progress():
    opt = _exposure_opt()
    progress = {"steps": 0, "tokens": 0}
    update_optimizer_exposure(progress, opt)
    progress["steps"] += 1
    snapshot = json.dumps(progress, sort_keys=True)
    for g in opt.param_groups:
        g["lr"] = float("nan")
    with pytest.raises(ValueError):
        update_optimizer_exposure(progress, opt)
    for g in opt.param_groups:
        g["lr"] = 1e308
        g["weight_decay"] = 1e308 if g["weight_decay"] else 0.0
    with pytest.raises(ValueError):  # lr * wd overflows
        update_optimizer_exposure(progress, opt)
    assert json.dumps(progress, sort_keys=True) == snapshot
    other = _exposure_opt()
    other.param_groups[0]["params"] = other.param_groups[0]["params"][:1]  # a different group identity
    for g in opt.param_groups:
        g["lr"], g["weight_decay"] = 0.01, (0.1 if g["weight_decay"] else 0.0)
    with pytest.raises(ValueError, match="not the group"):
        update_optimizer_exposure(progress, other)
    assert json.dumps(progress, sort_keys=True) == snapshot
    with pytest.raises(ValueError):
        update_optimizer_exposure({"steps": True, "tokens": 0}, opt)


def test_exposure_started_mid_run_is_not_a_complete_history():
    opt = _exposure_opt()
    progress = {"steps": 40, "tokens": 4000}  # a parent from before exposure was recorded
    update_optimizer_exposure(progress, opt)
    rec = progress["optimizer_exposure"]
    assert not rec["complete_history"] and rec["known_start_steps"] == 40 and rec["known_start_tokens"] == 4000
    progress["steps"] += 1
    update_optimizer_exposure(progress, opt)
    assert progress["optimizer_exposure"]["observed_steps"] == 2


def test_exposure_covers_both_muon_and_adamw_children():
    model = TensorLM(ModelConfig(**TINY_MODEL))
    opt = make_optimizer(model, TrainConfig(optimizer="muon", lr=0.02, aux_adamw_lr=0.003))
    exp = update_optimizer_exposure({"steps": 0, "tokens": 0}, opt)
    kinds = [g["identity"]["optimizer_kind"] for g in exp["groups"]]
    assert kinds[0] == "muon" and "adamw" in kinds


# --------------------------------------------------------------------------- throughput canary
def test_canary_passes_on_fast_updates_and_publishes(tmp_path):
    out = tmp_path / "canary.json"
    c = ThroughputCanary(2, 100.0, 1, output_path=out)
    c.observe({"step": 1, "prediction_tokens": 10, "seconds": 100.0})  # warm-up: ignored
    c.observe({"step": 2, "prediction_tokens": 1000, "seconds": 1.0})
    c.observe({"step": 3, "prediction_tokens": 1000, "seconds": 1.0})
    assert c.status == "passed" and c.require_complete()["tokens_per_second"] == 1000.0
    assert json.loads(out.read_text())["status"] == "passed"


def test_canary_fails_loudly_when_slow_or_incomplete(tmp_path):
    c = ThroughputCanary(1, 1e9, 0)
    with pytest.raises(RuntimeError):
        c.observe({"step": 1, "prediction_tokens": 10, "seconds": 1.0})
    assert c.status == "below_threshold"
    short = ThroughputCanary(3, 1.0, 0, output_path=tmp_path / "short.json")
    short.observe({"step": 1, "prediction_tokens": 10, "seconds": 1.0})
    with pytest.raises(RuntimeError):
        short.require_complete()
    assert json.loads((tmp_path / "short.json").read_text())["status"] == "insufficient"
    with pytest.raises(ValueError):
        ThroughputCanary(1, 1.0, 0).observe({"step": 0, "prediction_tokens": 1, "seconds": 1.0})
    with pytest.raises(FileExistsError):
        ThroughputCanary(1, 1.0, 0, output_path=tmp_path / "short.json")


def test_exposure_accepts_the_fused_adamw_kernel_optimizer():
    """The CUDA trainer's AdamW (the fused multi-tensor kernel subclass) has the same exposure
    record as torch's AdamW over the same groups."""
    from tensor_train_ing_b200.optim import FusedAdamW
    from tensor_train_ing_b200.train import optimizer_groups
    model = TensorLM(ModelConfig(**TINY_MODEL))
    plain = torch.optim.AdamW(optimizer_groups(model, 0.1), lr=0.01)
    fused = FusedAdamW(optimizer_groups(model, 0.1), lr=0.01)
    assert (update_optimizer_exposure({"steps": 0, "tokens": 0}, fused)
            == update_optimizer_exposure({"steps": 0, "tokens": 0}, plain))


def test_presets_count_the_parameters_the_benchmark_builds():
    """The planner's parameter counts are those of the modules the benchmark instantiates (meta-device
    blocks, never formulas): 2,018,084,864 for the 1B bench shape with its untied 50304-row vocabulary."""
    from tensor_train_ing_b200.models.shapes import count_params, preset
    cfg = preset("bench_1b", padded_vocab=50304, vocab_size=50257)
    c = count_params(cfg)
    assert c["total"] == 2018084864
    assert c["embedding"] == 2 * 50304 * 2048
    # per block: q1 k1 q2 k2 v o (6 d^2 at 16 x 128 = d) and L R D (3 d x 8192), plus norm vectors
    assert c["non_embedding"] == 24 * (6 * 2048 ** 2 + 3 * 2048 * 8192)
    assert c["total"] - c["embedding"] - c["non_embedding"] == 24 * (c["per_block"] - c["non_embedding"] // 24) + 2048


def test_memory_plan_layouts_and_the_gathered_weights():
    """Replicated state is 10 bytes per parameter; parameter sharding moves fp32 state to owners; the
    fused all-gather keeps 1/N of the bf16 rows plus the staging window, so the 32B plan on 8 GPUs
    shrinks by about 7/8 of the bf16 model."""
    from tensor_train_ing_b200.models.shapes import count_params, largest_weight_group, memory_plan, min_gpus, preset
    cfg = preset("bench_32b", loss_chunk_tokens=8192, activation_checkpointing=True)
    rep = memory_plan(cfg, gpus=8, micro_tokens_per_gpu=8192)
    shard = memory_plan(cfg, gpus=8, micro_tokens_per_gpu=8192, shard_params=True, fused_gather=False)
    gath = memory_plan(cfg, gpus=8, micro_tokens_per_gpu=8192, shard_params=True)
    assert not rep["fits"] and shard["fits"] and gath["fits"]
    assert gath["total_GB"] < shard["total_GB"] < rep["total_GB"]
    c = count_params(cfg)
    sharded = c["non_embedding"] + cfg.padded_vocab * cfg.d_model
    saved = 2 * sharded * 7 / 8 - 2 * 8 * largest_weight_group(cfg)
    assert abs((shard["total_GB"] - gath["total_GB"]) - saved / 1e9) < 0.2
    assert "gathered by the GEMMs" in gath["layout"]
    small = min_gpus(preset("bench_1b", loss_chunk_tokens=8192), 16384)
    assert small is not None and small["gpus"] == 1 and not small["shard_params"]


def test_parameter_sharding_is_chosen_by_size_or_forced(monkeypatch):
    from tensor_train_ing_b200.models.shapes import needs_parameter_sharding, preset
    monkeypatch.delenv("TTB_SHARD_PARAMS", raising=False)
    assert not needs_parameter_sharding(preset("bench_1b"), 8)
    assert needs_parameter_sharding(preset("bench_32b"), 8)
    assert not needs_parameter_sharding(preset("bench_32b"), 1)  # one rank cannot shard
    monkeypatch.setenv("TTB_SHARD_PARAMS", "1")
    assert needs_parameter_sharding(preset("bench_1b"), 2)
    monkeypatch.setenv("TTB_SHARD_PARAMS", "0")
    assert not needs_parameter_sharding(preset("bench_32b"), 8)


def test_selective_recompute_choice_fits_the_plan():
    """The automatic choice keeps as many blocks' activations as fit 92 % of the device after the
    checkpointed plan; a device with no room recomputes every block."""
    from tensor_train_ing_b200.models.shapes import blocks_to_recompute, memory_plan, preset
    cfg = preset("bench_7b", loss_chunk_tokens=8192, activation_checkpointing=True)
    total = 191.5e9  # a B200 as torch reports it
    n = blocks_to_recompute(cfg, gpus=1, micro_tokens_per_gpu=16384, device_bytes=total)
    kept = cfg.layers - n
    assert 0 < kept < cfg.layers
    assert memory_plan(cfg, gpus=1, micro_tokens_per_gpu=16384, kept_blocks=kept)["total_GB"] * 1e9 <= 0.92 * total
    assert memory_plan(cfg, gpus=1, micro_tokens_per_gpu=16384, kept_blocks=kept + 1)["total_GB"] * 1e9 > 0.92 * total
    assert blocks_to_recompute(cfg, gpus=8, micro_tokens_per_gpu=16384, device_bytes=total) < n  # sharded state frees room
    assert blocks_to_recompute(cfg, gpus=1, micro_tokens_per_gpu=16384, device_bytes=100e9) == cfg.layers
