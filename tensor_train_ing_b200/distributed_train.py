"""Distributed trainer: the serial trainer's update contract across ranks (reference
tnlm/distributed_train.py:45-550).

* Data: each rank reads its contiguous slice of one global packed-row stream (``RankPackedSampler``).
* Quotas: every micro-batch round the ranks exchange their valid-target counts; targets are kept in
  rank order until the update's ``global_prediction_tokens_per_update`` is reached (the rest are
  masked), so an update scores exactly the targets a serial run of the same stream would.
* Loss: every rank back-propagates ``local_sum / global_quota``; gradients are summed across ranks.
* Update: ``ShardedDataParallel`` reduce-scatters the gradients onto their owning ranks, the global
  norm is clipped (error on non-finite), each rank updates the matrices it owns and one all-gather
  returns the replicas to bitwise agreement.
* Lifecycle: collective lagged calibration and commits, TaperNorm, per-update score bounds (max over
  ranks) with batch-bound QK-clip (the reference refuses QK-clip in its distributed trainer,
  tnlm/distributed_train.py:126-128; here every rank clips each head by the maximum over the ranks of
  their last micro-batch's bound, so the replicated weights stay identical), constant / cooldown /
  cosine schedules, context forks, sharded
  recovery checkpoints (``ttb-sharded-v1``) and an optional full-state weight export.
* Control plane: validation and I/O run under ``_phase`` so a rank-local error fails every rank at
  the same step; time limits use the maximum over ranks so all ranks stop at the same update.
"""
from __future__ import annotations

import hashlib
import json
import shutil
import time
from functools import partial
from pathlib import Path

import torch
import torch.distributed as dist

from .budget import SpendLedger
from .calibration import _check_lagged_divisor, calibrate_lagged
from .checkpoint_plan import checkpoint_retention_policy
from .config import Config
from .distributed_checkpoint import (_agree, _phase, export_distributed_weights, is_distributed_checkpoint,
                                     load_distributed_checkpoint, read_distributed_manifest,
                                     save_distributed_checkpoint)
from .models.model import TensorLM
from .models.shapes import needs_parameter_sharding
from .models.normalization import lagged_modules, spectral_step
from .optimizer_exposure import update_optimizer_exposure
from .parallel.sharded import ShardedDataParallel
from .reference_dcp import (is_reference_checkpoint, load_reference_checkpoint, read_reference_manifest,
                            save_reference_checkpoint)
from .runtime import determinism_metadata, full_config, resume_validator, seed_all
from .schedules import lr_multiplier, schedule_multiplier, schedule_steps, validate_schedule
from .train import _mask_to_count, _validate_batch, make_optimizer
from .training_stability import BatchScoreBounds, StabilityPolicy
from .training_taper import TaperLifecycle, validate_taper_config


def _digest_words(hexdigest: str) -> list[int]:
    raw = bytes.fromhex(hexdigest)
    return [int.from_bytes(raw[i:i + 8], "little", signed=True) for i in range(0, 32, 8)]


def _words_digest(words) -> str:
    return b"".join(int(w).to_bytes(8, "little", signed=True) for w in words).hex()


CHECKPOINT_FORMATS = ("ttb-sharded-v1", "tnlm-dcp-v1")


def distributed_train_run(cfg, run_dir, *, max_steps, max_seconds, device="cuda", resume=None, cooldown_steps=None,
                          cooldown_end_tokens=None, run_budget_usd=None, export_max_state_bytes=None,
                          context_fork=False, checkpoint_format="ttb-sharded-v1"):
    """Train up to ``max_steps`` new updates on every rank of the initialised process group.

    ``resume`` may name a checkpoint of either sharded format; ``checkpoint_format`` chooses the
    format of the checkpoints this run writes (``tnlm-dcp-v1`` is the reference's, which its own
    distributed trainer resumes)."""
    from .data import RankPackedSampler, batch_hash, manifest_hash as hash_manifest
    if not dist.is_initialized():
        raise ValueError("distributed_train_run requires an initialized process group")
    if isinstance(cfg, (str, Path)):
        cfg = Config.from_yaml(str(cfg))
    rank, world = dist.get_rank(), dist.get_world_size()
    project, data = cfg.raw.get("project", {}), cfg.raw.get("data", {})
    _agree("distributed launch request", {"config": full_config(cfg), "max_steps": max_steps,
                                          "max_seconds": max_seconds, "resume": str(resume) if resume else None,
                                          "cooldown_steps": cooldown_steps, "cooldown_end_tokens": cooldown_end_tokens,
                                          "context_fork": context_fork, "export": export_max_state_bytes,
                                          "run_dir": str(Path(run_dir).resolve())})
    planned_total = schedule_steps(cfg.train.rung_total_tokens, cfg.train.global_prediction_tokens_per_update)

    def preflight():
        if type(context_fork) is not bool or (context_fork and resume is None):
            raise ValueError("context_fork must be Boolean and requires an explicit parent checkpoint")
        if cfg.train.schedule == "cosine" and cooldown_end_tokens is not None:
            raise ValueError("cosine does not support a separate cooldown")
        validate_schedule(cfg.train.schedule, planned_total, cooldown_steps=cooldown_steps)
        if validate_taper_config(cfg):
            if round(cfg.train.taper_end_fraction * planned_total) <= validate_schedule(cfg.train.schedule, planned_total):
                raise ValueError("TaperNorm endpoint must be strictly after positive warmup_steps")
        if StabilityPolicy.from_config(cfg).clipping and StabilityPolicy.from_config(cfg).clip_source != "batch_bound":
            raise ValueError("distributed QK-clip supports qk_clip_source='batch_bound' only")
        if StabilityPolicy.from_config(cfg).stability_every:
            raise ValueError("periodic stability logging supports serial training only")
        if export_max_state_bytes is not None and (type(export_max_state_bytes) is not int or export_max_state_bytes <= 0):
            raise ValueError("export_max_state_bytes must be a positive integer or None")
        if max_steps <= 0 or max_seconds <= 0:
            raise ValueError("positive max_steps/max_seconds required")
        if cooldown_steps is not None and (type(cooldown_steps) is not int or cooldown_steps <= 0 or resume is None):
            raise ValueError("cooldown requires positive cooldown_steps and an explicit parent checkpoint")
        if cooldown_end_tokens is not None and (type(cooldown_end_tokens) is not int or cooldown_end_tokens <= 0
                                                or cooldown_steps is None):
            raise ValueError("cooldown_end_tokens requires a positive integer and cooldown_steps")
        if resume is not None and not (is_distributed_checkpoint(resume) or is_reference_checkpoint(resume)):
            raise ValueError("distributed resume needs a sharded checkpoint of the same world size")
        if checkpoint_format not in CHECKPOINT_FORMATS:
            raise ValueError(f"checkpoint_format must be one of {CHECKPOINT_FORMATS}")
        dev = torch.device(device)
        if dev.type == "cuda" and not torch.cuda.is_available():
            raise RuntimeError("CUDA requested but unavailable")
        rate = project.get("gpu_hourly_rate_usd")
        if rate is None or (dev.type == "cuda" and rate <= 0):
            raise ValueError("declare actual gpu_hourly_rate_usd (explicit 0 allowed for CPU)")
        return float(rate)
    rate = _phase("distributed preflight", preflight)
    if project.get("dry_run", True):
        return {"dry_run": True, "world_size": world, "planned_steps": planned_total, "context_fork": context_fork,
                "parent": str(resume) if resume else None}
    dev = torch.device(device)
    run_dir = Path(run_dir)
    parent_manifest = None
    old_context = data.get("context", 512)
    if resume is not None:
        parent_manifest = _phase("parent manifest", lambda: (read_reference_manifest(resume)
                                                             if is_reference_checkpoint(resume)
                                                             else read_distributed_manifest(resume)))
        _phase("parent config validation", lambda: resume_validator(cfg, context_fork=context_fork)(parent_manifest["config"]))
        old_context = parent_manifest["config"].get("data", {}).get("context", 512)
    ledger = SpendLedger(project.get("spend_ledger", "runs/spend.json"), project.get("total_budget_usd", 1000),
                         project.get("reserve_usd", 150), stage_budgets=project.get("stage_budgets")) if rank == 0 else None
    run_id = str(run_dir.resolve())

    def fresh():
        if run_dir.exists():
            raise FileExistsError(f"run directory already exists: {run_dir}")

    def begin():
        if rank == 0:
            # one reservation for the whole job: the declared rate is per GPU
            ledger.begin(run_id, rate * world, max_seconds, run_budget_usd, parent_checkpoint=resume,
                         cost_margin_fraction=project.get("cost_margin_fraction", .1), stage=project.get("stage", "A"))
            run_dir.mkdir(parents=True)
    # every rank looks for an existing directory before rank 0 creates it (one phase each: a rank that
    # looked after the creation would otherwise refuse the job's own directory)
    _phase("run directory check", fresh)
    _phase("run reservation", begin)
    started = time.monotonic()
    status = "failed"

    def max_value(value: float) -> float:
        t = torch.tensor([float(value)], dtype=torch.float64, device=dev if dist.get_backend() == "nccl" else "cpu")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def max_over_ranks_(t: torch.Tensor) -> None:
        on = t.to(dev) if dist.get_backend() == "nccl" else t
        dist.all_reduce(on, op=dist.ReduceOp.MAX)
        if on is not t:
            t.copy_(on.cpu())

    def expired() -> bool:
        return max_value(time.monotonic() - started) >= max_seconds

    try:
        def build():
            sampler = RankPackedSampler(data["manifest"], rank=rank, world_size=world, split="train",
                                        batch_size=data.get("micro_batch_size", 1), context=old_context,
                                        seed=cfg.train.seed)
            tokenizer = sampler.manifest["tokenizer"]
            if tokenizer.get("test_only") and dev.type != "cpu":
                raise ValueError("test-only tokenizer manifests are restricted to CPU fixtures")
            seed_all(cfg.train.seed)
            shard = needs_parameter_sharding(cfg.model, world, dev)
            if shard:  # built from the streamed serial initialisation: no rank holds all fp32 weights
                with torch.device("meta"):
                    model = TensorLM(cfg.model)
            else:
                model = TensorLM(cfg.model).to(dev)
            fused = dev.type == "cuda" and model.fused_path_supported()[0]
            dp = ShardedDataParallel(model, dev, fused=fused, shard_params=shard)
            optimizer = make_optimizer(model, cfg.train, only=dp.owned_ids())
            # the logical (unsharded) optimizer: never stepped, it carries the full group structure
            # for exposure bookkeeping, which must not depend on which rank owns what
            logical = make_optimizer(model, cfg.train)
            if len(logical.param_groups) != len(optimizer.param_groups):
                raise ValueError("sharded and logical optimizer group structures differ")
            return sampler, model, dp, optimizer, logical
        sampler, model, dp, optimizer, logical = _phase("model and sampler construction", build)
        manifest_hash = hash_manifest(data["manifest"])
        _agree("data identity", manifest_hash)
        _agree("initial replicas", hashlib.sha256(b"".join(
            v.detach().cpu().contiguous().view(-1).view(torch.uint8).numpy().tobytes()[:4096]
            for _, v in sorted(dp.replicated_state().items()))).hexdigest())
        progress = {"steps": 0, "tokens": 0, "scheduler_step": 0, "input_tokens_seen": 0,
                    "discarded_prediction_targets": 0, "world_size": world,
                    "warmup_steps": validate_schedule(cfg.train.schedule, planned_total)}
        parent = None
        previous = {}
        if resume is not None:
            loader = (partial(load_reference_checkpoint, logical=logical) if is_reference_checkpoint(resume)
                      else load_distributed_checkpoint)
            loaded = loader(resume, model, optimizer, sampler, dp, expected_manifest_hash=manifest_hash,
                            config_validator=resume_validator(cfg, context_fork=context_fork))
            progress.update(loaded["progress"])
            if loaded.get("config_compatibility", {}).get("defaulted_fields"):
                progress.setdefault("config_compatibility_history", []).append(
                    {"checkpoint": str(Path(resume).resolve()), **loaded["config_compatibility"]})
            progress["world_size"] = world
            previous = progress.get("distributed_schedule", {}) or {}
            parent = {"path": str(Path(resume).resolve()),
                      "manifest_sha256": hashlib.sha256((Path(resume) / "manifest.json").read_bytes()).hexdigest()}
            if previous.get("cooldown_steps") is not None and cooldown_steps != previous["cooldown_steps"]:
                raise ValueError("cooled checkpoint requires explicit matching cooldown_steps")
            if context_fork:
                from .runtime import record_context_fork
                source_state = sampler.state_dict()["stream"]
                forked = sampler.fork_context(data.get("context", 512))
                sampler = forked
                record_context_fork(progress, old_context=old_context, new_context=data.get("context", 512),
                                    parent=parent, source_state=source_state)
        else:
            progress["batch_history"] = [{"batch_tokens": cfg.train.global_prediction_tokens_per_update,
                                          "lr": cfg.train.lr, "aux_adamw_lr": cfg.train.aux_adamw_lr,
                                          "start_tokens": 0, "start_step": 0, "source": "fresh"}]
            progress["context_history"] = [{"context": data.get("context", 512), "start_tokens": 0, "start_step": 0,
                                            "source": "fresh"}]
        branch_base = previous.get("branch_base_lr") or [g.get("base_lr", g["lr"]) for g in optimizer.param_groups]
        if cooldown_steps is not None and previous.get("cooldown_steps") is None:
            progress["scheduler_step"] = 0
            progress["cooldown_start_tokens"] = progress["tokens"]
        progress["distributed_schedule"] = {"cooldown_steps": cooldown_steps, "branch_base_lr": branch_base}
        norms = lagged_modules(model)
        if norms and resume is None:
            calibration = calibrate_lagged(model, cfg, data["manifest"], dev, deadline=started + max_seconds,
                                           collective_control=True)
            progress["calibration"] = _agree("calibration report", calibration)
        for norm in norms:
            _phase("lagged divisor validation", lambda norm=norm: _check_lagged_divisor(norm))
        taper = TaperLifecycle(model, cfg, total_steps=planned_total, warmup_steps=progress["warmup_steps"],
                              distributed=True)
        taper.before_step(progress["steps"])
        taper.set_valid_mask(None)
        bounds = BatchScoreBounds(model, cfg)
        policy = StabilityPolicy.from_config(cfg)
        clip_tau, clip_every = policy.clip_tau, policy.clip_every
        token_limit = (progress["cooldown_start_tokens"] + cooldown_steps * cfg.train.global_prediction_tokens_per_update
                       if cooldown_steps is not None else cfg.train.rung_total_tokens)
        if cooldown_end_tokens is not None:
            if not token_limit - cfg.train.global_prediction_tokens_per_update < cooldown_end_tokens <= token_limit:
                raise ValueError("cooldown endpoint must match the cooldown step horizon")
            token_limit = progress["cooldown_end_tokens"] = cooldown_end_tokens
        retention = checkpoint_retention_policy(cfg)
        keep_recovery = retention["keep_recovery_checkpoints"]
        every = int(project.get("checkpoint_every_steps", 0))

        def save(name):
            if checkpoint_format == "tnlm-dcp-v1":
                return save_reference_checkpoint(run_dir / name, model, optimizer, sampler, dp, logical=logical,
                                                 config=full_config(cfg), progress=progress,
                                                 manifest_hash=manifest_hash, parent=parent)
            return save_distributed_checkpoint(run_dir / name, model, optimizer, sampler, dp,
                                               config=full_config(cfg), progress=progress, manifest_hash=manifest_hash,
                                               parent=parent,
                                               extra={"cooldown_steps": cooldown_steps,
                                                      "cooldown_end_tokens": cooldown_end_tokens,
                                                      "runtime": {"determinism": determinism_metadata(),
                                                                  "device": str(dev), "world_size": world}})
        rolling, history = [], []
        stop_reason = "max_steps"
        model.train()
        for _ in range(max_steps):
            if expired():
                stop_reason = "runtime_cap"
                break
            if progress["tokens"] >= token_limit:
                stop_reason = "token_limit"
                break
            step_started = time.monotonic()
            taper.before_step(progress["steps"])
            if bounds.enabled:
                bounds.begin_update()
            sched = progress["scheduler_step"]
            mult = (lr_multiplier(sched, planned_total, cooldown_steps=cooldown_steps) if cooldown_steps is not None
                    else schedule_multiplier(sched, planned_total, schedule=cfg.train.schedule,
                                             warmup_steps=progress["warmup_steps"]))
            for group, base in zip(optimizer.param_groups, branch_base):
                group["lr"] = (base if cooldown_steps is not None else group.get("base_lr", cfg.train.lr)) * mult
            dp.zero_grad()
            spectral_step(model)
            wanted = min(cfg.train.global_prediction_tokens_per_update, token_limit - progress["tokens"])
            accumulated, local_loss, local_anchor, inputs, discarded, rounds, empty = 0, 0.0, 0.0, 0, 0, [], 0
            while accumulated < wanted:
                if expired():
                    raise TimeoutError("runtime cap during accumulation; recover from the last complete checkpoint")

                def next_batch():
                    batch = sampler.next_batch()
                    _validate_batch(*batch, cfg.model.vocab_size)
                    return batch
                batch = _phase("batch validation", next_batch)
                idx, docs, targets = batch
                raw = int((targets != -100).sum())
                mine = torch.tensor([raw, *_digest_words(batch_hash(batch))], dtype=torch.int64,
                                    device=dev if dist.get_backend() == "nccl" else "cpu")
                table = torch.empty(world * 5, dtype=torch.int64, device=mine.device)
                dist.all_gather_into_tensor(table, mine)
                table = table.view(world, 5).cpu().tolist()
                counts = [row[0] for row in table]
                remaining = wanted - accumulated
                quotas = [max(0, min(c, remaining - sum(counts[:i]))) for i, c in enumerate(counts)]
                selected = quotas[rank]
                targets = _mask_to_count(targets, selected)
                discarded += raw - selected
                inputs += int((docs >= 0).sum())
                rounds.append({"raw_counts": counts, "selected_counts": quotas,
                               "batch_hashes": [_words_digest(row[1:]) for row in table]})
                if not sum(quotas):
                    empty += 1
                    if empty > 100:
                        raise ValueError("no valid prediction targets in the global stream")
                    continue
                empty = 0
                idx, docs, targets = (t.to(dev, non_blocking=True) for t in (idx, docs, targets))
                if taper.enabled:
                    taper.set_valid_mask((docs >= 0) if taper.collecting else (targets != -100))
                for norm in norms:
                    norm.collecting = True
                    norm.set_valid_mask(docs >= 0)
                try:
                    def forward_backward():
                        _, loss, n = model(idx, doc_ids=docs, targets=targets, reduction="sum")
                        if bounds.enabled:
                            bounds.observe()
                        if int(n) != selected or not bool(torch.isfinite(loss)):
                            raise FloatingPointError("invalid loss/count; update aborted")
                        objective = loss / wanted
                        anchor = taper.anchor() if taper.enabled else None
                        extra = 0.0
                        if anchor is not None:
                            if not bool(torch.isfinite(anchor)):
                                raise FloatingPointError("non-finite TaperNorm anchor")
                            objective = objective + taper.anchor_lambda * anchor * (selected / wanted)
                            extra = float(anchor.detach()) * selected
                        objective.backward()
                        dp.after_backward()
                        return float(loss.detach()), extra
                    loss_value, anchor_value = _phase("forward/backward", forward_backward)
                finally:
                    taper.set_valid_mask(None)
                    for norm in norms:
                        norm.collecting = False
                        norm.set_valid_mask(None)
                local_loss += loss_value
                local_anchor += anchor_value
                accumulated += sum(quotas)
            score_bound_max = max_value(bounds.finish_update()) if bounds.enabled else None
            dp.reduce_gradients()
            norm_value = dp.clip_(cfg.train.grad_clip)
            grad_norm = float(norm_value)
            if grad_norm != grad_norm or grad_norm in (float("inf"), float("-inf")):
                raise FloatingPointError(f"non-finite global gradient norm {grad_norm}")
            optimizer.step()
            dp.gather_params()
            for norm in norms:
                norm.commit()
                _phase("lagged divisor validation", lambda norm=norm: _check_lagged_divisor(norm))
            totals = torch.tensor([local_loss, inputs, discarded, local_anchor], dtype=torch.float64,
                                  device=dev if dist.get_backend() == "nccl" else "cpu")
            dist.all_reduce(totals)
            totals = totals.cpu().tolist()
            for lg, g in zip(logical.param_groups, optimizer.param_groups):
                lg["lr"] = g["lr"]
            update_optimizer_exposure(progress, logical)
            progress["steps"] += 1
            progress["tokens"] += accumulated
            progress["scheduler_step"] = sched + 1
            progress["input_tokens_seen"] += int(totals[1])
            progress["discarded_prediction_targets"] += int(totals[2])
            taper.after_step(progress["steps"])
            clipping = None
            if clip_tau > 0 and progress["steps"] % clip_every == 0:
                bounds.reduce_last(max_over_ranks_)  # one clip factor per head on every rank
                clipping = bounds.clip(clip_tau)
                if dp.shard_params:
                    dp.gather_params()  # owners rescaled their masters: refresh every rank's copies
            seconds = max_value(time.monotonic() - step_started)
            elapsed = max_value(time.monotonic() - started)
            record = {"step": progress["steps"], "tokens": progress["tokens"], "prediction_tokens": accumulated,
                      "loss": totals[0] / accumulated, "grad_norm": grad_norm, "lr": optimizer.param_groups[0]["lr"],
                      "optimizer_group_lrs": [g["lr"] for g in optimizer.param_groups], "rounds": rounds,
                      "seconds": seconds, "run_elapsed_seconds": elapsed,
                      "run_billed_usd": elapsed * rate * world / 3600, "world_size": world,
                      "tokens_per_second": accumulated / seconds if seconds > 0 else None}
            record.update(taper.metrics(totals[3] / accumulated))
            if score_bound_max is not None:
                record["score_bound_max"] = score_bound_max
            if clipping is not None:
                record["qk_clip"] = clipping
            history.append(record)

            def log():
                if rank == 0:
                    with open(run_dir / "metrics.jsonl", "a") as out:
                        out.write(json.dumps(record, allow_nan=False) + "\n")
            _phase("metrics append", log)
            if keep_recovery and every > 0 and progress["steps"] % every == 0:
                rolling.append(run_dir / f"recovery-{progress['steps']:08d}")
                save(rolling[-1].name)
                while len(rolling) > keep_recovery:
                    old = rolling.pop(0)
                    _phase("recovery retention", lambda old=old: shutil.rmtree(old) if rank == 0 else None)
        final = save("final")
        export = None
        if export_max_state_bytes is not None:
            export = export_distributed_weights(run_dir / "final-weights", model, config=full_config(cfg),
                                                progress=progress, manifest_hash=manifest_hash,
                                                parent={"path": str((run_dir / "final").resolve())},
                                                max_state_bytes=export_max_state_bytes, dp=dp)
        result = {"checkpoint": str((run_dir / "final").resolve()), "checkpoint_manifest": final,
                  "weights_export": export, "progress": progress, "history": history[-1000:],
                  "stop_reason": stop_reason, "world_size": world, "run_id": run_id,
                  "metrics_path": str(run_dir / "metrics.jsonl"),
                  "parameters": model.param_counts(), "operator_audit": model.operator_audit(),
                  "ownership": {"shard_elements": dp.shard,
                                "owned_parameters_per_rank": [sum(1 for u in dp.layout if u["owner"] == r)
                                                              for r in range(world)]}}

        def write_result():
            if rank == 0:
                (run_dir / "result.json").write_text(json.dumps(result, indent=2, default=str))
        _phase("result publication", write_result)
        status = "complete"
        return result
    finally:
        if rank == 0:
            ledger.finish(run_id, time.monotonic() - started, status)
