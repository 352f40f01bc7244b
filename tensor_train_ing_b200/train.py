"""Serial trainer: token-quota updates, explicit cooldowns and local cost accounting.

Semantics of the reference serial trainer (tnlm/train.py:168-685): each optimizer update collects
exactly ``global_prediction_tokens_per_update`` valid targets from the packed sampler (overflow
targets of the last micro-batch are masked, rows without targets are omitted), backpropagates
the summed loss, divides gradients by the valid-target count, clips the global norm
(error on non-finite), steps the optimizer, then runs the lagged/taper/spectral lifecycle,
QK-clip and the stability probe at their cadences, writes one ``metrics.jsonl`` row, and saves
milestone / recovery / final checkpoints in the reference's format.  Resumes continue bit-exactly
(RNG, sampler cursor, optimizer state); cooldowns, context forks and batch branches fork a
parent checkpoint into a new run directory.

On CUDA the model runs on the fused sm_100a path; weight gradients accumulate in fp32 directly
inside the GEMM epilogues.
"""
from __future__ import annotations

import hashlib
import json
import math
import os
import shutil
import time
from collections import deque
from contextlib import nullcontext
from pathlib import Path

import torch

from .batch_branch import BatchBranch, segment
from .budget import SpendLedger
from .calibration import _check_lagged_divisor, calibrate_lagged
from .checkpoint_plan import checkpoint_retention_policy, checkpoint_storage_plan, pending_milestone_tokens
from .checkpoint_storage import require_checkpoint_space
from .config import Config
from .models.model import TensorLM
from .models.normalization import lagged_modules, spectral_step
from .optim import hidden_matrix
from .optimizer_exposure import update_optimizer_exposure
from .runtime import determinism_metadata, full_config, resume_validator, seed_all, training_execution
from .schedules import lr_multiplier, schedule_multiplier, schedule_steps, validate_schedule
from .training_stability import BatchScoreBounds, StabilityPolicy, TrainingStabilityProbe
from .training_taper import TaperLifecycle, validate_taper_config


def _assert_no_analysis_state(model):
    for name, module in model.named_modules():
        if getattr(module, "ablate", frozenset()):
            raise RuntimeError(f"analysis ablation leaked into training: {name}")
        if any(getattr(module, f, None) is not None for f in ("denom_mode", "denom_saved", "denom_const")):
            raise RuntimeError(f"analysis denominator state leaked into training: {name}")


def optimizer_groups(model, weight_decay):
    vocab = {id(model.embed.weight), id(model.unembed.weight)}
    decay, no_decay = [], []
    for name, p in model.named_parameters():
        if p.requires_grad:
            (decay if hidden_matrix(name, p) and id(p) not in vocab else no_decay).append(p)
    return [{"params": decay, "weight_decay": weight_decay}, {"params": no_decay, "weight_decay": 0.0}]


def make_optimizer(model, cfg):
    """Trainer optimizer: plain reference AdamW grouping, or the scaling/Muon builder."""
    if cfg.optimizer == "muon" or getattr(getattr(model, "cfg", None), "width_scaling_base", None) is not None:
        from .optim import make_optimizer as scaling_optimizer
        return scaling_optimizer(model, cfg)
    if cfg.optimizer != "adamw":
        raise ValueError("optimizer must be adamw or muon")
    fused = torch.cuda.is_available() and all(p.is_cuda for p in model.parameters())
    return torch.optim.AdamW(optimizer_groups(model, cfg.weight_decay_hidden), lr=cfg.lr,
                             betas=(cfg.beta1, cfg.beta2), fused=fused or None)


def plan_search(cfg) -> dict:
    project, data = cfg.raw.get("project", {}), cfg.raw.get("data", {})
    if cfg.train.rung_total_tokens <= 0 or cfg.train.global_prediction_tokens_per_update <= 0:
        raise ValueError("positive rung/token batch required for planning")
    planned = schedule_steps(cfg.train.rung_total_tokens, cfg.train.global_prediction_tokens_per_update)
    warmup = validate_schedule(cfg.train.schedule, planned)
    ledger = SpendLedger(project.get("spend_ledger", "runs/spend.json"), project.get("total_budget_usd", 1000),
                         project.get("reserve_usd", 150), stage_budgets=project.get("stage_budgets"))
    stage = project.get("stage", "A")
    if stage not in ledger.stage_budgets:
        raise ValueError(f"unknown budget stage: {stage}")
    throughput = project.get("measured_prediction_tokens_per_second")
    if throughput is not None:
        throughput = float(throughput)
        if not math.isfinite(throughput) or throughput <= 0:
            raise ValueError("measured throughput must be finite and positive")
    setup = float(project.get("estimated_setup_seconds", 0))
    if not math.isfinite(setup) or setup < 0:
        raise ValueError("estimated setup time must be finite and nonnegative")
    seconds = cfg.train.rung_total_tokens / throughput + setup if throughput is not None else None
    rate = project.get("gpu_hourly_rate_usd")
    if rate is not None:
        rate = float(rate)
        if not math.isfinite(rate) or rate < 0:
            raise ValueError("hourly rate must be finite and nonnegative")
    snap = json.loads(ledger.path.read_text()) if ledger.path.exists() else {"runs": {}}
    rows = list(snap["runs"].values())
    spent = lambda pred: sum(r.get("spent_usd", 0) + r.get("reserved_usd", 0) for r in rows if pred(r))  # noqa: E731
    return {"dry_run": project.get("dry_run", True), "manifest": data.get("manifest"),
            "context": data.get("context", 512), "tokens": cfg.train.rung_total_tokens,
            "prediction_tokens_per_update": cfg.train.global_prediction_tokens_per_update,
            "normalization": cfg.model.normalization, "optimizer": cfg.train.optimizer, "schedule": cfg.train.schedule,
            "checkpoint_storage_plan": checkpoint_storage_plan(cfg), "rate_usd_per_hour": project.get("gpu_hourly_rate_usd"),
            "total_budget_usd": project.get("total_budget_usd", 1000), "reserve_usd": project.get("reserve_usd", 150),
            "stage": stage, "stage_budgets_usd": ledger.stage_budgets,
            "unallocated_project_usd": ledger.total - spent(lambda r: True),
            "unallocated_regular_usd": ledger.total - ledger.reserve - spent(lambda r: r.get("stage", "A") != "Reserve"),
            "unallocated_stage_usd": ledger.stage_budgets[stage] - spent(lambda r: r.get("stage", "A") == stage),
            "cost_margin_fraction": project.get("cost_margin_fraction", .1), "warmup_steps": warmup,
            "planned_optimizer_steps": planned, "warmup_dominates_rung": warmup > .1 * planned,
            "proposed_runs": [{"normalization": cfg.model.normalization, "tokens": cfg.train.rung_total_tokens,
                               "projected_seconds": seconds,
                               "projected_usd": seconds * rate / 3600 if seconds is not None and rate is not None else None}],
            "note": "one configured trajectory; projected cost needs measured valid-target throughput and actual hourly rate"}


def _mask_to_count(targets, count):
    targets = targets.clone()
    positions = (targets.flatten() != -100).nonzero().flatten()
    targets.flatten()[positions[count:]] = -100
    return targets


def _trim_unscored_rows(idx, docs, targets, *, enabled, bucket_rows=False):
    """Drop rows without any scored target (their loss is zero).  ``bucket_rows`` keeps the row
    count to one of a few sizes by retaining original zero-loss rows."""
    if not enabled:
        return idx, docs, targets
    keep = (targets != -100).any(dim=1)
    if bool(keep.all()):
        return idx, docs, targets
    if bucket_rows:
        scored = int(keep.sum())
        if scored:
            rows = idx.shape[0]
            sizes = sorted({1, *((rows + d - 1) // d for d in (8, 4, 2, 1))})
            target = next(s for s in sizes if s >= scored)
            if target == rows:
                return idx, docs, targets
            extra = target - scored
            if extra:
                keep[(~keep).nonzero().flatten()[:extra]] = True
    return idx[keep], docs[keep], targets[keep]


def _validate_batch(idx, docs, targets, vocab):
    if (idx < 0).any() or (idx >= vocab).any():
        raise ValueError("input token outside real vocabulary")
    if ((docs < 0) & (targets != -100)).any():
        raise ValueError("padded-token targets must be -100")
    if ((targets != -100) & ((targets < 0) | (targets >= vocab))).any():
        raise ValueError("target outside real vocabulary")


@training_execution()
def train_run(cfg, run_dir, *, max_steps, max_seconds, device="cuda", resume=None, cooldown_steps=None,
              cooldown_end_tokens=None, run_budget_usd=None, context_fork=False, batch_tokens=None, lr_scale=None,
              _step_profiler=None, _throughput_canary=None):
    """Run a bounded trajectory into a new run directory (resume also forks into a new directory)."""
    if type(context_fork) is not bool or (context_fork and resume is None):
        raise ValueError("context_fork requires a Boolean flag and explicit parent checkpoint")
    if isinstance(cfg, (str, Path)):
        cfg = Config.from_yaml(str(cfg))
    parent_cfg = cfg
    branch = BatchBranch.request(cfg, batch_tokens=batch_tokens, lr_scale=lr_scale, resume=resume,
                                 context_fork=context_fork, cooldown_steps=cooldown_steps)
    if branch is not None:
        cfg = branch.child_config(cfg)
    batch_change = branch.record() if branch is not None else None
    parent_validator = resume_validator(parent_cfg, context_fork=context_fork)
    retention = checkpoint_retention_policy(cfg)
    policy = StabilityPolicy.from_config(cfg)
    stability_every, clip_tau, clip_every, clip_source = (policy.stability_every, policy.clip_tau,
                                                          policy.clip_every, policy.clip_source)
    planned_total = schedule_steps(cfg.train.rung_total_tokens, cfg.train.global_prediction_tokens_per_update)
    if validate_taper_config(cfg):
        if round(cfg.train.taper_end_fraction * planned_total) <= validate_schedule(cfg.train.schedule, planned_total):
            raise ValueError("TaperNorm endpoint must be strictly after positive warmup_steps")
    if cfg.train.schedule == "cosine" and cooldown_end_tokens is not None:
        raise ValueError("cosine does not support a separate cooldown")
    validate_schedule(cfg.train.schedule, planned_total, cooldown_steps=cooldown_steps)
    if cfg.raw.get("project", {}).get("dry_run", True):
        return {**plan_search(cfg), "batch_branch": batch_change, "context_fork": context_fork,
                "new_context": cfg.raw.get("data", {}).get("context", 512),
                "parent": str(resume) if resume is not None else None,
                "parent_validation": "pending" if resume is not None else None}
    world = int(os.environ.get("WORLD_SIZE", "1"))
    active = torch.distributed.get_world_size() if torch.distributed.is_available() and torch.distributed.is_initialized() else 1
    if max(world, active) > 1:
        raise RuntimeError("train_run supports one process; use distributed_train_run for several ranks")
    from .checkpoint import _digest, load_checkpoint, save_checkpoint, verified_state_path
    from .data import PackedSampler, batch_hash, manifest_hash as hash_manifest

    project, data = cfg.raw.get("project", {}), cfg.raw.get("data", {})
    if type(cfg.model.loss_chunk_tokens) is not int or cfg.model.loss_chunk_tokens < 0:
        raise ValueError("loss_chunk_tokens must be a nonnegative integer")
    if cooldown_steps is not None and (cooldown_steps <= 0 or resume is None):
        raise ValueError("cooldown requires positive cooldown_steps and an explicit parent checkpoint")
    if cooldown_end_tokens is not None and (type(cooldown_end_tokens) is not int or cooldown_end_tokens <= 0
                                            or cooldown_steps is None):
        raise ValueError("cooldown_end_tokens requires a positive integer and cooldown_steps")
    history_limit = int(project.get("history_limit", 1000))
    if history_limit <= 0:
        raise ValueError("history_limit must be positive; full metrics persist in metrics.jsonl")
    if max_steps <= 0 or max_seconds <= 0:
        raise ValueError("positive max_steps/max_seconds required")
    if data.get("document_boundary_mask", True) is not True or data.get("reset_position_at_document", True) is not True:
        raise ValueError("this reference requires document masking and reset positions")
    if not cfg.train.fp32_optimizer_state or not cfg.train.fp32_norm_reductions:
        raise ValueError("reference requires FP32 optimizer state and norm reductions")
    dev = torch.device(device)
    if dev.type == "cuda" and not torch.cuda.is_available():
        raise RuntimeError("CUDA requested but unavailable")
    rate = project.get("gpu_hourly_rate_usd")
    if rate is None or (dev.type == "cuda" and rate <= 0):
        raise ValueError("declare actual gpu_hourly_rate_usd (explicit 0 allowed for CPU)")
    run_dir = Path(run_dir)
    if run_dir.exists():
        raise FileExistsError(f"run directory already exists: {run_dir}")
    if _throughput_canary is not None:
        _throughput_canary.bind_output(run_dir / "canary.json")
    if resume is None:
        require_checkpoint_space(run_dir.parent, checkpoint_storage_plan(cfg, max_steps=max_steps)["required_additional_bytes"])
    old_context = data.get("context", 512)
    if resume is not None:
        saved = torch.load(verified_state_path(resume), map_location="cpu", weights_only=False, mmap=True)
        parent_validator(saved["config"])
        if branch is not None:
            branch.check_parent(saved, cfg)
        old_context = saved["config"].get("data", {}).get("context", 512)
        del saved
    ledger = SpendLedger(project.get("spend_ledger", "runs/spend.json"), project.get("total_budget_usd", 1000),
                         project.get("reserve_usd", 150), stage_budgets=project.get("stage_budgets"))
    run_id = str(run_dir.resolve())
    ledger.begin(run_id, rate, max_seconds, run_budget_usd, parent_checkpoint=resume,
                 cost_margin_fraction=project.get("cost_margin_fraction", .1), stage=project.get("stage", "A"))
    started = time.monotonic()
    status = "failed"
    try:
        sampler = PackedSampler(data["manifest"], split="train", batch_size=data.get("micro_batch_size", 1),
                                context=old_context, seed=cfg.train.seed)
        manifest_hash = hash_manifest(data["manifest"])
        tokenizer = sampler.manifest["tokenizer"]
        if tokenizer.get("test_only") and dev.type != "cpu":
            raise ValueError("test-only tokenizer manifests are restricted to CPU fixtures")
        if data.get("tokenizer") is not None and data["tokenizer"] not in (tokenizer["name"], tokenizer.get("fingerprint_sha256")):
            raise ValueError("configured tokenizer does not match immutable manifest")
        run_dir.mkdir(parents=True)
        seed_all(cfg.train.seed)
        if dev.type == "cuda":
            torch.cuda.reset_peak_memory_stats(dev)
        model = TensorLM(cfg.model).to(dev)
        _assert_no_analysis_state(model)
        optimizer = make_optimizer(model, cfg.train)
        progress = {"steps": 0, "tokens": 0, "skipped_updates": [], "scheduler_step": 0, "input_tokens_seen": 0,
                    "discarded_prediction_targets": 0,
                    "warmup_steps": validate_schedule(cfg.train.schedule, planned_total)}
        parent = None
        resume_extra = {}
        if resume:
            payload = load_checkpoint(resume, model, optimizer, sampler, expected_manifest_hash=manifest_hash,
                                      config_validator=parent_validator, map_location="cpu")
            progress.update(payload["progress"])
            if payload.get("config_compatibility", {}).get("defaulted_fields"):
                progress.setdefault("config_compatibility_history", []).append(
                    {"checkpoint": str(Path(resume).resolve()), **payload["config_compatibility"]})
            parent = {"path": str(Path(resume).resolve()),
                      "manifest_sha256": hashlib.sha256((Path(resume) / "manifest.json").read_bytes()).hexdigest()}
            if branch is not None:
                branch.check_parent(payload, cfg)
                branch.apply(optimizer, sampler, progress, parent_cfg, cfg, parent)
                import yaml
                (run_dir / "branch-config.yaml").write_text(yaml.safe_dump(full_config(cfg), sort_keys=False))
            if context_fork:
                from .runtime import record_context_fork
                source_state = sampler.state_dict()
                sampler = sampler.fork_context(data.get("context", 512))
                record_context_fork(progress, old_context=old_context, new_context=data.get("context", 512),
                                    parent=parent, source_state=source_state)
            if payload.get("extra", {}).get("cooldown_steps") is not None and cooldown_steps is None:
                raise ValueError("cooldown checkpoint requires explicit matching cooldown_steps")
            resume_extra = payload.get("extra", {}) or {}
            del payload
        else:
            progress["batch_history"] = [segment(cfg, tokens=0, steps=0, source="fresh")]
            progress["context_history"] = [{"context": data.get("context", 512), "start_tokens": 0, "start_step": 0,
                                            "source": "fresh"}]
        branch_base_lr = [g["lr"] for g in optimizer.param_groups]
        if cooldown_steps is not None:
            prev = resume_extra.get("cooldown_steps")
            if prev is not None:
                if prev != cooldown_steps:
                    raise ValueError("cannot change an existing cooldown horizon")
                if cooldown_end_tokens != resume_extra.get("cooldown_end_tokens"):
                    raise ValueError("cannot change an existing cooldown endpoint")
                branch_base_lr = resume_extra["branch_base_lr"]
            else:
                progress["scheduler_step"] = 0
                progress["cooldown_start_tokens"] = progress["tokens"]
        norms = lagged_modules(model)
        if norms and not resume:
            progress["calibration"] = calibrate_lagged(model, cfg, data["manifest"], dev, deadline=started + max_seconds)
        for norm in norms:
            _check_lagged_divisor(norm)
        bounds = BatchScoreBounds(model, cfg)
        forward = model  # the fused sm_100a path is the compiled path; no tracing compiler is used
        total_steps = planned_total
        if cooldown_steps is not None:
            token_limit = progress["cooldown_start_tokens"] + cooldown_steps * cfg.train.global_prediction_tokens_per_update
            if cooldown_end_tokens is not None:
                lower = token_limit - cfg.train.global_prediction_tokens_per_update
                if not lower < cooldown_end_tokens <= token_limit:
                    raise ValueError("cooldown endpoint must match the cooldown step horizon")
                token_limit = cooldown_end_tokens
                progress["cooldown_end_tokens"] = cooldown_end_tokens
        else:
            token_limit = cfg.train.rung_total_tokens
        storage_plan = checkpoint_storage_plan(cfg, start_tokens=progress["tokens"], token_limit=token_limit,
                                               max_steps=max_steps, cooldown=cooldown_steps is not None)
        admission = require_checkpoint_space(run_dir, storage_plan["required_additional_bytes"])
        (run_dir / "checkpoint_storage_plan.json").write_text(
            json.dumps({"plan": storage_plan, "admission": admission}, indent=2, allow_nan=False) + "\n")
        taper = TaperLifecycle(model, cfg, total_steps=total_steps, warmup_steps=progress["warmup_steps"])
        taper.before_step(progress["steps"])
        taper.set_valid_mask(None)

        def save(name):
            save_checkpoint(run_dir / name, model, optimizer, sampler, config=full_config(cfg), progress=progress,
                            manifest_hash=manifest_hash, parent=parent,
                            extra={"operator_audit": model.operator_audit(), "cooldown_steps": cooldown_steps,
                                   "cooldown_end_tokens": cooldown_end_tokens, "branch_base_lr": branch_base_lr,
                                   "runtime": {"determinism": determinism_metadata(), "device": str(dev),
                                               "fused_sm100a_path": model.uses_fused_path(torch.empty(1, device=dev)),
                                               "autocast_enabled": False,
                                               "compute_dtype": "bfloat16" if dev.type == "cuda" else "float32"}})
            return run_dir / name

        t0 = time.monotonic()
        if retention["save_initial_checkpoint"]:
            save("initial")
        ckpt_seconds = 3 * (time.monotonic() - t0) if retention["save_initial_checkpoint"] else 0.0
        probe = TrainingStabilityProbe(cfg, dev) if stability_every or (clip_tau > 0 and clip_source == "probe") else None
        last_recovery = time.monotonic()
        rolling = deque()
        milestones = list(pending_milestone_tokens(cfg, start_tokens=progress["tokens"], token_limit=token_limit,
                                                   reachable_tokens=storage_plan["reachable_tokens"],
                                                   include_branch=cooldown_steps is None and cfg.train.schedule != "cosine"))
        history = deque(maxlen=history_limit)
        prev_log_tokens, prev_log_elapsed = progress["tokens"], 0.0
        slowest = 0.0
        new_updates = warm_updates = 0
        model.train()
        empty_batches = 0
        every = int(project.get("checkpoint_every_steps", 0))
        every_seconds = float(project.get("checkpoint_every_seconds", 300))
        keep_recovery = retention["keep_recovery_checkpoints"]
        if every_seconds <= 0:
            raise ValueError("checkpoint interval must be positive")
        stop_reason = "max_steps"
        region = getattr(_step_profiler, "region", lambda _name: nullcontext())
        for local_step in range(max_steps):
            _assert_no_analysis_state(model)
            elapsed = time.monotonic() - started
            if elapsed >= max_seconds or elapsed + slowest + ckpt_seconds >= max_seconds:
                stop_reason = "runtime_cap"
                break
            if progress["tokens"] >= token_limit:
                stop_reason = "token_limit"
                break
            step_start = time.monotonic()
            if _step_profiler is not None:
                _step_profiler.start_step(local_step)
            bounds.begin_update()
            taper.before_step(progress["steps"])
            sched_step = progress.get("scheduler_step", progress["steps"])
            mult = (lr_multiplier(sched_step, total_steps, cooldown_steps=cooldown_steps) if cooldown_steps is not None
                    else schedule_multiplier(sched_step, total_steps, schedule=cfg.train.schedule,
                                             warmup_steps=progress["warmup_steps"]))
            for group, base in zip(optimizer.param_groups, branch_base_lr):
                group["lr"] = (base if cooldown_steps is not None else group.get("base_lr", cfg.train.lr)) * mult
            optimizer.zero_grad(set_to_none=True)
            with region("tnlm.spectral_step"):
                spectral_step(model)
            wanted = min(cfg.train.global_prediction_tokens_per_update, token_limit - progress["tokens"])
            valid_total, loss_total, hashes = 0, 0.0, []
            anchor_total = 0.0
            positions, omitted = 0, 0
            while valid_total < wanted:
                if time.monotonic() - started >= max_seconds:
                    raise TimeoutError("runtime cap during accumulation; last complete checkpoint is recoverable")
                with region("tnlm.sampler"):
                    batch = sampler.next_batch()
                with region("tnlm.prepare_batch"):
                    if "context_fork_exposure" in progress:
                        for k, v in sampler.batch_context_exposure().items():
                            progress["context_fork_exposure"][k] += v
                    idx, docs, targets = batch
                    _validate_batch(idx, docs, targets, cfg.model.vocab_size)
                    raw_valid = int((targets != -100).sum())
                    targets = _mask_to_count(targets, wanted - valid_total)
                    progress["input_tokens_seen"] += int((docs >= 0).sum())
                    n = int((targets != -100).sum())
                    progress["discarded_prediction_targets"] += raw_valid - n
                    if not n:
                        empty_batches += 1
                        if empty_batches > 100:
                            raise ValueError("no valid prediction targets in sampler")
                        continue
                    empty_batches = 0
                    hashes.append(batch_hash(batch))
                    rows = idx.shape[0]
                    idx, docs, targets = _trim_unscored_rows(idx, docs, targets,
                                                             enabled=not norms and not taper.enabled)
                    omitted += rows - idx.shape[0]
                    positions += idx.numel()
                with region("tnlm.transfer"):
                    idx, docs, targets = (t.to(dev, non_blocking=True) for t in (idx, docs, targets))
                if taper.enabled:
                    taper.set_valid_mask((docs >= 0) if taper.collecting else (targets != -100))
                for norm in norms:
                    norm.collecting = True
                    norm.set_valid_mask(docs >= 0)
                try:
                    with region("tnlm.forward"):
                        _, loss, actual_n = forward(idx, doc_ids=docs, targets=targets, reduction="sum")
                    if bounds.enabled:
                        bounds.observe()
                    anchor = taper.anchor()
                    objective = loss if anchor is None else loss + taper.anchor_lambda * anchor * n
                    if anchor is not None:
                        anchor_total += float(anchor.detach()) * n
                    with region("tnlm.validate_loss"):
                        if int(actual_n) != n or not torch.isfinite(objective):
                            raise FloatingPointError("invalid loss/count; update aborted")
                    with region("tnlm.backward"):
                        objective.backward()
                finally:
                    taper.set_valid_mask(None)
                    for norm in norms:
                        norm.collecting = False
                        norm.set_valid_mask(None)
                valid_total += n
                with region("tnlm.loss_accounting"):
                    loss_total += float(loss.detach())
            score_bound_max = bounds.finish_update() if bounds.enabled else None
            with region("tnlm.optimizer"):
                grads = [p.grad for p in model.parameters() if p.grad is not None]
                torch._foreach_div_(grads, float(valid_total))
                grad_norm = torch.nn.utils.clip_grad_norm_(model.parameters(), cfg.train.grad_clip,
                                                           error_if_nonfinite=True)
                optimizer.step()
            update_optimizer_exposure(progress, optimizer)
            for norm in norms:
                norm.commit()
                _check_lagged_divisor(norm)
            if dev.type == "cuda":
                with region("tnlm.synchronize"):
                    torch.cuda.synchronize(dev)
            progress["steps"] += 1
            taper.after_step(progress["steps"])
            progress["tokens"] += valid_total
            progress["scheduler_step"] = sched_step + 1
            new_updates += 1
            warm_updates += int(cooldown_steps is None and sched_step < progress["warmup_steps"])
            clipping = stability = None
            if clip_tau > 0 and progress["steps"] % clip_every == 0:
                with region("tnlm.qk_clip"):
                    clipping = bounds.clip(clip_tau) if clip_source == "batch_bound" else probe.clip(model, clip_tau)
            if stability_every and progress["steps"] % stability_every == 0:
                with region("tnlm.stability_probe"):
                    stability = probe.sample(model)
            now = time.monotonic()
            record = {"step": progress["steps"], "tokens": progress["tokens"], "prediction_tokens": valid_total,
                      "loss": loss_total / valid_total, "grad_norm": float(grad_norm),
                      "optimizer_group_lrs": [g["lr"] for g in optimizer.param_groups],
                      "optimizer_exposure": progress["optimizer_exposure"], "lr": optimizer.param_groups[0]["lr"],
                      "batch_hashes": hashes, "microbatches": len(hashes), "forward_input_positions": positions,
                      "unscored_rows_omitted": omitted, "seconds": now - step_start,
                      "run_elapsed_seconds": now - started, "run_billed_usd": (now - started) * rate / 3600}
            record["tokens_per_second"] = ((record["tokens"] - prev_log_tokens)
                                           / (record["run_elapsed_seconds"] - prev_log_elapsed))
            prev_log_tokens, prev_log_elapsed = record["tokens"], record["run_elapsed_seconds"]
            record.update(taper.metrics(anchor_total / valid_total))
            if score_bound_max is not None:
                record["score_bound_max"] = score_bound_max
            if clipping is not None:
                record["qk_clip"] = clipping
            if stability is not None:
                record["stability"] = stability
            if _step_profiler is not None:
                _step_profiler.finish_step()
            slowest = max(slowest, time.monotonic() - step_start)
            history.append(record)
            with open(run_dir / "metrics.jsonl", "a") as out:
                out.write(json.dumps(record, allow_nan=False) + "\n")
            if _throughput_canary is not None:
                _throughput_canary.observe(record)
            while milestones and progress["tokens"] >= milestones[0]:
                save(f"milestone-{milestones.pop(0):012d}")
            due = ((every > 0 and progress["steps"] % every == 0)
                   or time.monotonic() - last_recovery >= max(every_seconds, 20 * ckpt_seconds))
            if keep_recovery and due:
                t0 = time.monotonic()
                rolling.append(save(f"recovery-{progress['steps']:08d}"))
                ckpt_seconds = time.monotonic() - t0
                last_recovery = time.monotonic()
                while len(rolling) > keep_recovery:
                    candidate = rolling.popleft()
                    with ledger.locked() as led:
                        refs = {r.get("parent_checkpoint") for r in led["runs"].values()}
                        if str(candidate.resolve()) not in refs:
                            shutil.rmtree(candidate)
        if _throughput_canary is not None:
            _throughput_canary.require_complete()
        final = save("final")
        from .evaluate import _training_descriptor
        descriptor = _training_descriptor({"config": full_config(cfg), "progress": progress,
                                           "extra": {"cooldown_steps": cooldown_steps,
                                                     "cooldown_end_tokens": cooldown_end_tokens}})
        result = {"training_descriptor": descriptor, "batch_branch": batch_change, "checkpoint": str(final),
                  "checkpoint_storage_plan": storage_plan, "checkpoint_storage_admission": admission,
                  "progress": progress, "history": list(history), "metrics_path": str(run_dir / "metrics.jsonl"),
                  "spend_ledger": str(ledger.path.resolve()), "run_id": run_id, "parent": parent,
                  "history_limit": history_limit,
                  "cuda_peak_allocated_bytes": torch.cuda.max_memory_allocated(dev) if dev.type == "cuda" else None,
                  "cuda_peak_reserved_bytes": torch.cuda.max_memory_reserved(dev) if dev.type == "cuda" else None,
                  "operator_audit": model.operator_audit(), "parameters": model.param_counts(),
                  "runtime": {"determinism": determinism_metadata(), "device": str(dev), "torch": str(torch.__version__),
                              "bf16_compute": cfg.train.bf16_compute and dev.type == "cuda"},
                  "model_config": full_config(cfg)["model"], "train_config": full_config(cfg)["train"],
                  "data": {"manifest_sha256": manifest_hash, "context": data.get("context", 512), "tokenizer": tokenizer},
                  "stop_reason": stop_reason, "compile_enabled": False, "warmup_steps": progress["warmup_steps"],
                  "warmup_fraction_of_completed_updates": warm_updates / new_updates if new_updates else None,
                  "warmup_dominates_completed_segment": warm_updates > .1 * new_updates,
                  "lagged_collection_policy": "all nonpadding tokens; once per optimizer step",
                  "elapsed_seconds_before_final_accounting": time.monotonic() - started}
        if _throughput_canary is not None:
            result["throughput_canary"] = _throughput_canary.report()
        if _step_profiler is not None:
            result["kernel_profile"] = _step_profiler.report()
        (run_dir / "result.json").write_text(json.dumps(result, indent=2))
        status = "complete"
        return result
    finally:
        try:
            if _step_profiler is not None:
                _step_profiler.close()
        finally:
            ledger.finish(run_id, time.monotonic() - started, status)


def profile_run(cfg, run_dir, *, steps, warmup_steps=2, max_seconds, device="cuda", run_budget_usd=None,
                kernels=False, trace_steps=0) -> dict:
    """Measure complete training steps (declared warm-up excluded) with optional kernel profiles."""
    if isinstance(cfg, (str, Path)):
        cfg = Config.from_yaml(str(cfg))
    if steps <= 0 or warmup_steps < 0:
        raise ValueError("positive timed steps and nonnegative warmup_steps required")
    if type(trace_steps) is not int or not 0 <= trace_steps <= 100:
        raise ValueError("trace_steps must be an integer in [0, 100]")
    if kernels and torch.device(device).type != "cuda":
        raise ValueError("kernel profiling requires a CUDA device")
    from .profiling import KernelProfile
    profiler = (KernelProfile(warmup_steps, trace_dir=Path(run_dir) / "traces", trace_steps=max(1, trace_steps),
                              cuda=torch.device(device).type == "cuda", kernels=kernels)
                if kernels or trace_steps else None)
    result = train_run(cfg, run_dir, max_steps=steps + warmup_steps, max_seconds=max_seconds, device=device,
                       run_budget_usd=run_budget_usd, **({"_step_profiler": profiler} if profiler else {}))
    if result.get("dry_run"):
        return {**result, "command": "profile", "warmup_steps": warmup_steps, "timed_steps": steps,
                "kernels": kernels, "trace_steps": trace_steps}
    timed_s = tokens = timed = observed = micro = fwd = omitted = 0
    metrics = Path(result["metrics_path"])
    if metrics.exists():
        for i, line in enumerate(metrics.read_text().splitlines()):
            rec = json.loads(line)
            observed += 1
            if i >= warmup_steps:
                timed += 1
                timed_s += rec["seconds"]
                tokens += rec["prediction_tokens"]
                micro += rec["microbatches"]
                fwd += rec["forward_input_positions"]
                omitted += rec["unscored_rows_omitted"]
    report = {"command": "profile", "device": str(device), "determinism": result.get("runtime", {}).get("determinism"),
              "kernels": kernels, "trace_steps": trace_steps, "requested_timed_steps": steps,
              "completed_timed_steps": timed, "warmup_steps": warmup_steps, "completed_total_steps": observed,
              "timed_training_seconds": timed_s, "timed_prediction_tokens": tokens, "timed_microbatches": micro,
              "timed_forward_input_positions": fwd, "timed_unscored_rows_omitted": omitted,
              "forward_positions_per_prediction_target": fwd / tokens if tokens else None,
              "mean_microbatches_per_step": micro / timed if timed else None,
              "prediction_tokens_per_second": tokens / timed_s if timed_s > 0 else None,
              "mean_training_step_seconds": timed_s / timed if timed else None,
              "cuda_peak_allocated_bytes": result["cuda_peak_allocated_bytes"],
              "cuda_peak_reserved_bytes": result["cuda_peak_reserved_bytes"], "checkpoint": result["checkpoint"],
              "operator_audit": result["operator_audit"], "parameters": result["parameters"],
              "compile_enabled": result["compile_enabled"], "stop_reason": result["stop_reason"],
              "note": "step timers include batch preparation, forward/backward and optimizer work; checkpoint saves, "
                      "metric writes and profiler finalization are outside step timers"}
    if profiler is not None:
        report["kernel_profile"] = result["kernel_profile"]
    ledger = Path(cfg.raw.get("project", {}).get("spend_ledger", "runs/spend.json"))
    report["billing"] = json.loads(ledger.read_text())["runs"][str(Path(run_dir).resolve())]
    (Path(run_dir) / "profile.json").write_text(json.dumps(report, indent=2, allow_nan=False))
    return report
