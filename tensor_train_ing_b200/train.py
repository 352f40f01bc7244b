"""Serial trainer: token-quota updates, explicit cooldowns and local cost accounting.

The update contract is the reference serial trainer's (tnlm/train.py:168-685): each optimizer
update collects exactly ``global_prediction_tokens_per_update`` valid targets from the packed
sampler (targets past the quota in the last micro-batch are masked, rows left without targets are
dropped when that cannot change any statistic), back-propagates each micro-batch's summed loss,
divides the accumulated gradients by the update's target count, clips the global norm (an error
if it is not finite), steps the optimizer, then runs the lagged / taper / spectral lifecycle,
QK-clip and the stability probe at their cadences, appends one ``metrics.jsonl`` row and saves
milestone, recovery and final checkpoints in the shared format.  Runs resume bit-exactly (RNG,
sampler cursor, optimizer state); cooldowns, context forks and batch branches fork a parent
checkpoint into a new run directory.

The pieces: ``QuotaBatcher`` turns sampler rows into the micro-batches of one update;
``TrainEngine`` runs forward / backward / update on them (the fused sm_100a path on CUDA, where
weight gradients accumulate in fp32 inside the GEMM epilogues and AdamW is one multi-tensor
kernel per group); ``CheckpointSchedule`` decides and performs the saves; ``MetricsLog`` writes
the rows; ``train_run`` validates a ``RunRequest`` and drives ``_Run``.
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
from dataclasses import dataclass
from pathlib import Path
from typing import Callable

import torch

from .batch_branch import BatchBranch, segment
from .budget import SpendLedger
from .calibration import _check_lagged_divisor, calibrate_lagged
from .checkpoint_plan import checkpoint_retention_policy, checkpoint_storage_plan, pending_milestone_tokens
from .checkpoint_storage import require_checkpoint_space
from .config import Config
from .engine import TrainEngine
from .models.model import TensorLM
from .models.normalization import lagged_modules, spectral_step
from .optim import FusedAdamW, hidden_matrix
from .optimizer_exposure import update_optimizer_exposure
from .runtime import determinism_metadata, full_config, resume_validator, seed_all, training_execution
from .schedules import lr_multiplier, schedule_multiplier, schedule_steps, validate_schedule
from .training_stability import BatchScoreBounds, StabilityPolicy, TrainingStabilityProbe
from .training_taper import TaperLifecycle, validate_taper_config

MAX_EMPTY_BATCHES = 100


# ====================================================================================== optimizer
def optimizer_groups(model, weight_decay, only: set[int] | None = None):
    """The reference's plain AdamW grouping: decay on block matrices, none on the vocabulary
    matrices and small parameters, each group in parameter order (the checkpointed optimizer layout
    depends on it).  ``only``: keep these parameter ids (a rank's owned parameters); both groups
    are kept even when empty."""
    vocab = {id(model.embed.weight), id(model.unembed.weight)}
    decay, plain = [], []
    for name, p in model.named_parameters():
        if p.requires_grad and (only is None or id(p) in only):
            (decay if hidden_matrix(name, p) and id(p) not in vocab else plain).append(p)
    return [{"params": decay, "weight_decay": weight_decay}, {"params": plain, "weight_decay": 0.0}]


def make_optimizer(model, cfg, only: set[int] | None = None):
    """The trainers' optimizer: plain AdamW grouping (the fused multi-tensor kernel on CUDA), or
    the width-scaling / Muon builder.  ``only``: over a rank's owned parameters, with the same groups."""
    if cfg.optimizer == "muon" or getattr(getattr(model, "cfg", None), "width_scaling_base", None) is not None:
        from .optim import make_optimizer as scaling_optimizer
        return scaling_optimizer(model, cfg, only=only)
    if cfg.optimizer != "adamw":
        raise ValueError("optimizer must be adamw or muon")
    groups = optimizer_groups(model, cfg.weight_decay_hidden, only)
    params = [p for g in groups for p in g["params"]]
    if params and all(p.is_cuda for p in params):
        return FusedAdamW(groups, lr=cfg.lr, betas=(cfg.beta1, cfg.beta2))
    return torch.optim.AdamW(groups, lr=cfg.lr, betas=(cfg.beta1, cfg.beta2))


# ====================================================================================== planning
def _ledger_for(project) -> SpendLedger:
    return SpendLedger(project.get("spend_ledger", "runs/spend.json"), project.get("total_budget_usd", 1000),
                       project.get("reserve_usd", 150), stage_budgets=project.get("stage_budgets"))


def _checked_number(value, what, *, positive=False):
    """None, or ``value`` as a finite float that is nonnegative (positive if asked)."""
    if value is None:
        return None
    value = float(value)
    if not math.isfinite(value) or value < 0 or (positive and value == 0):
        raise ValueError(f"{what} must be finite and {'positive' if positive else 'nonnegative'}")
    return value


def plan_search(cfg) -> dict:
    """The dry-run plan of one configured trajectory: steps, warm-up, storage, budget headroom and,
    given a measured throughput and an hourly rate, its projected time and cost."""
    project, data, train = cfg.raw.get("project", {}), cfg.raw.get("data", {}), cfg.train
    if train.rung_total_tokens <= 0 or train.global_prediction_tokens_per_update <= 0:
        raise ValueError("positive rung/token batch required for planning")
    planned = schedule_steps(train.rung_total_tokens, train.global_prediction_tokens_per_update)
    warmup = validate_schedule(train.schedule, planned)
    ledger = _ledger_for(project)
    stage = project.get("stage", "A")
    if stage not in ledger.stage_budgets:
        raise ValueError(f"unknown budget stage: {stage}")
    throughput = _checked_number(project.get("measured_prediction_tokens_per_second"), "measured throughput",
                                 positive=True)
    setup = _checked_number(project.get("estimated_setup_seconds", 0), "estimated setup time")
    rate = _checked_number(project.get("gpu_hourly_rate_usd"), "hourly rate")
    seconds = train.rung_total_tokens / throughput + setup if throughput is not None else None
    rows = list((json.loads(ledger.path.read_text()) if ledger.path.exists() else {"runs": {}})["runs"].values())

    def held(keep):
        return sum(r.get("spent_usd", 0) + r.get("reserved_usd", 0) for r in rows if keep(r))
    return {"dry_run": project.get("dry_run", True), "manifest": data.get("manifest"),
            "context": data.get("context", 512), "tokens": train.rung_total_tokens,
            "prediction_tokens_per_update": train.global_prediction_tokens_per_update,
            "normalization": cfg.model.normalization, "optimizer": train.optimizer, "schedule": train.schedule,
            "checkpoint_storage_plan": checkpoint_storage_plan(cfg), "rate_usd_per_hour": project.get("gpu_hourly_rate_usd"),
            "total_budget_usd": project.get("total_budget_usd", 1000), "reserve_usd": project.get("reserve_usd", 150),
            "stage": stage, "stage_budgets_usd": ledger.stage_budgets,
            "unallocated_project_usd": ledger.total - held(lambda r: True),
            "unallocated_regular_usd": ledger.total - ledger.reserve - held(lambda r: r.get("stage", "A") != "Reserve"),
            "unallocated_stage_usd": ledger.stage_budgets[stage] - held(lambda r: r.get("stage", "A") == stage),
            "cost_margin_fraction": project.get("cost_margin_fraction", .1), "warmup_steps": warmup,
            "planned_optimizer_steps": planned, "warmup_dominates_rung": warmup > .1 * planned,
            "proposed_runs": [{"normalization": cfg.model.normalization, "tokens": train.rung_total_tokens,
                               "projected_seconds": seconds,
                               "projected_usd": seconds * rate / 3600 if seconds is not None and rate is not None else None}],
            "note": "one configured trajectory; projected cost needs measured valid-target throughput and actual hourly rate"}


# ====================================================================================== batches
def _mask_to_count(targets, count):
    """A copy of ``targets`` that keeps only the first ``count`` valid targets (row-major order)."""
    targets = targets.clone()
    flat = targets.view(-1)
    flat[(flat != -100).nonzero().view(-1)[count:]] = -100
    return targets


def _trim_unscored_rows(idx, docs, targets, *, enabled, bucket_rows=False):
    """Drop rows without any scored target (their loss is zero).  ``bucket_rows`` rounds the kept
    row count up to one of a few sizes by keeping some zero-loss rows, so shapes repeat."""
    if not enabled:
        return idx, docs, targets
    keep = (targets != -100).any(dim=1)
    if bool(keep.all()):
        return idx, docs, targets
    if bucket_rows:
        scored = int(keep.sum())
        if scored:
            rows = idx.shape[0]
            size = next(s for s in sorted({1, *((rows + k - 1) // k for k in (8, 4, 2, 1))}) if s >= scored)
            if size == rows:
                return idx, docs, targets
            keep[(~keep).nonzero().view(-1)[:size - scored]] = True
    return idx[keep], docs[keep], targets[keep]


def _validate_batch(idx, docs, targets, vocab):
    if (idx < 0).any() or (idx >= vocab).any():
        raise ValueError("input token outside real vocabulary")
    if ((docs < 0) & (targets != -100)).any():
        raise ValueError("padded-token targets must be -100")
    if ((targets != -100) & ((targets < 0) | (targets >= vocab))).any():
        raise ValueError("target outside real vocabulary")


class QuotaBatcher:
    """The micro-batches of one update: sampler rows until ``wanted`` valid targets are collected.
    After the iteration, ``hashes``, ``positions`` and ``omitted`` describe the update."""

    def __init__(self, sampler, vocab, progress, *, trim_rows, region):
        self.sampler, self.vocab, self.progress = sampler, vocab, progress
        self.trim_rows, self.region = trim_rows, region
        self.empty_in_a_row = 0
        self.hashes, self.positions, self.omitted = [], 0, 0

    def _take(self, wanted_now):
        """The next sampler row batch masked to at most ``wanted_now`` targets, or None if it has none."""
        from .data import batch_hash
        progress = self.progress
        if "context_fork_exposure" in progress:
            for k, v in self.sampler.batch_context_exposure().items():
                progress["context_fork_exposure"][k] += v
        idx, docs, targets = self._batch
        _validate_batch(idx, docs, targets, self.vocab)
        offered = int((targets != -100).sum())
        targets = _mask_to_count(targets, wanted_now)
        progress["input_tokens_seen"] += int((docs >= 0).sum())
        n = int((targets != -100).sum())
        progress["discarded_prediction_targets"] += offered - n
        if not n:
            self.empty_in_a_row += 1
            if self.empty_in_a_row > MAX_EMPTY_BATCHES:
                raise ValueError("no valid prediction targets in sampler")
            return None
        self.empty_in_a_row = 0
        self.hashes.append(batch_hash(self._batch))
        rows = idx.shape[0]
        idx, docs, targets = _trim_unscored_rows(idx, docs, targets, enabled=self.trim_rows)
        self.omitted += rows - idx.shape[0]
        self.positions += idx.numel()
        return idx, docs, targets, n

    def micro_batches(self, wanted, deadline):
        """Yields (idx, docs, targets, valid targets) until ``wanted`` targets have been yielded."""
        self.hashes, self.positions, self.omitted = [], 0, 0
        collected = 0
        while collected < wanted:
            if time.monotonic() >= deadline:
                raise TimeoutError("runtime cap during accumulation; last complete checkpoint is recoverable")
            with self.region("tnlm.sampler"):
                self._batch = self.sampler.next_batch()
            with self.region("tnlm.prepare_batch"):
                taken = self._take(wanted - collected)
            if taken is None:
                continue
            collected += taken[3]
            yield taken


# ====================================================================================== saves and rows
class CheckpointSchedule:
    """Initial, milestone, rolling recovery and final checkpoints of a run.  A recovery checkpoint
    that a spend-ledger row names as its parent is never pruned."""

    def __init__(self, save: Callable, *, retention, milestones, every_steps, every_seconds, ledger):
        if every_seconds <= 0:
            raise ValueError("checkpoint interval must be positive")
        self.save = save
        self.keep = retention["keep_recovery_checkpoints"]
        self.save_initial = retention["save_initial_checkpoint"]
        self.milestones = list(milestones)
        self.every_steps, self.every_seconds, self.ledger = every_steps, every_seconds, ledger
        self.rolling: deque = deque()
        self.seconds_per_save = 0.0  # the run stops early enough to leave room for one more save
        self.last_recovery = time.monotonic()

    def initial(self):
        if self.save_initial:
            t0 = time.monotonic()
            self.save("initial")
            self.seconds_per_save = 3 * (time.monotonic() - t0)  # a trained checkpoint holds optimizer state too
        self.last_recovery = time.monotonic()

    def _prune(self):
        while len(self.rolling) > self.keep:
            oldest = self.rolling.popleft()
            with self.ledger.locked() as led:
                pinned = {r.get("parent_checkpoint") for r in led["runs"].values()}
                if str(oldest.resolve()) not in pinned:
                    shutil.rmtree(oldest)

    def after_update(self, progress):
        while self.milestones and progress["tokens"] >= self.milestones[0]:
            self.save(f"milestone-{self.milestones.pop(0):012d}")
        due = ((self.every_steps > 0 and progress["steps"] % self.every_steps == 0)
               or time.monotonic() - self.last_recovery >= max(self.every_seconds, 20 * self.seconds_per_save))
        if self.keep and due:
            t0 = time.monotonic()
            self.rolling.append(self.save(f"recovery-{progress['steps']:08d}"))
            self.seconds_per_save = time.monotonic() - t0
            self.last_recovery = time.monotonic()
            self._prune()


class MetricsLog:
    """``metrics.jsonl`` rows (the last ``limit`` also kept in memory), with run time, billed cost
    and the token rate since the previous row."""

    def __init__(self, path: Path, limit: int, started: float, rate: float, start_tokens: int):
        self.path, self.started, self.rate = path, started, rate
        self.history: deque = deque(maxlen=limit)
        self._last = (start_tokens, 0.0)

    def stamp(self, record: dict, now: float) -> dict:
        elapsed = now - self.started
        record["run_elapsed_seconds"] = elapsed
        record["run_billed_usd"] = elapsed * self.rate / 3600
        tokens0, elapsed0 = self._last
        record["tokens_per_second"] = (record["tokens"] - tokens0) / (elapsed - elapsed0)
        self._last = (record["tokens"], elapsed)
        return record

    def append(self, record: dict):
        self.history.append(record)
        with open(self.path, "a") as out:
            out.write(json.dumps(record, allow_nan=False) + "\n")


# ====================================================================================== the request
@dataclass
class RunRequest:
    """A validated trainer invocation: the (possibly branched) config and the fork parameters."""
    cfg: Config
    parent_cfg: Config
    branch: BatchBranch | None
    validator: Callable
    resume: object
    context_fork: bool
    cooldown_steps: int | None
    cooldown_end_tokens: int | None
    planned_total: int
    policy: StabilityPolicy

    @property
    def cooling(self) -> bool:
        return self.cooldown_steps is not None


def _request(cfg, *, resume, cooldown_steps, cooldown_end_tokens, context_fork, batch_tokens, lr_scale) -> RunRequest:
    """Checks that need no data or device; a dry run returns its plan after these."""
    if type(context_fork) is not bool or (context_fork and resume is None):
        raise ValueError("context_fork requires a Boolean flag and explicit parent checkpoint")
    if isinstance(cfg, (str, Path)):
        cfg = Config.from_yaml(str(cfg))
    parent_cfg = cfg
    branch = BatchBranch.request(cfg, batch_tokens=batch_tokens, lr_scale=lr_scale, resume=resume,
                                 context_fork=context_fork, cooldown_steps=cooldown_steps)
    if branch is not None:
        cfg = branch.child_config(cfg)
    validator = resume_validator(parent_cfg, context_fork=context_fork)
    checkpoint_retention_policy(cfg)
    policy = StabilityPolicy.from_config(cfg)
    planned = schedule_steps(cfg.train.rung_total_tokens, cfg.train.global_prediction_tokens_per_update)
    if validate_taper_config(cfg) and round(cfg.train.taper_end_fraction * planned) <= validate_schedule(
            cfg.train.schedule, planned):
        raise ValueError("TaperNorm endpoint must be strictly after positive warmup_steps")
    if cfg.train.schedule == "cosine" and cooldown_end_tokens is not None:
        raise ValueError("cosine does not support a separate cooldown")
    validate_schedule(cfg.train.schedule, planned, cooldown_steps=cooldown_steps)
    return RunRequest(cfg, parent_cfg, branch, validator, resume, context_fork, cooldown_steps, cooldown_end_tokens,
                      planned, policy)


def _check_launch(req: RunRequest, run_dir: Path, max_steps, max_seconds, device):
    """Everything that must hold before a ledger row is reserved; returns (device, hourly rate)."""
    cfg = req.cfg
    world = int(os.environ.get("WORLD_SIZE", "1"))
    active = (torch.distributed.get_world_size()
              if torch.distributed.is_available() and torch.distributed.is_initialized() else 1)
    if max(world, active) > 1:
        raise RuntimeError("train_run supports one process; use distributed_train_run for several ranks")
    project, data = cfg.raw.get("project", {}), cfg.raw.get("data", {})
    if type(cfg.model.loss_chunk_tokens) is not int or cfg.model.loss_chunk_tokens < 0:
        raise ValueError("loss_chunk_tokens must be a nonnegative integer")
    if req.cooling and (req.cooldown_steps <= 0 or req.resume is None):
        raise ValueError("cooldown requires positive cooldown_steps and an explicit parent checkpoint")
    end = req.cooldown_end_tokens
    if end is not None and (type(end) is not int or end <= 0 or not req.cooling):
        raise ValueError("cooldown_end_tokens requires a positive integer and cooldown_steps")
    if int(project.get("history_limit", 1000)) <= 0:
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
    if run_dir.exists():
        raise FileExistsError(f"run directory already exists: {run_dir}")
    return dev, rate


def _first_context(req: RunRequest) -> int:
    """The context of the run's first rows: the parent's when resuming (a fork changes it after
    the parent state is loaded).  Also validates the parent's config before any spend."""
    from .checkpoint import verified_state_path
    if req.resume is None:
        return req.cfg.raw.get("data", {}).get("context", 512)
    saved = torch.load(verified_state_path(req.resume), map_location="cpu", weights_only=False, mmap=True)
    req.validator(saved["config"])
    if req.branch is not None:
        req.branch.check_parent(saved, req.cfg)
    return saved["config"].get("data", {}).get("context", 512)


# ====================================================================================== entry point
@training_execution()
def train_run(cfg, run_dir, *, max_steps, max_seconds, device="cuda", resume=None, cooldown_steps=None,
              cooldown_end_tokens=None, run_budget_usd=None, context_fork=False, batch_tokens=None, lr_scale=None,
              _step_profiler=None, _throughput_canary=None):
    """Run a bounded trajectory into a new run directory (a resume also forks into a new directory)."""
    req = _request(cfg, resume=resume, cooldown_steps=cooldown_steps, cooldown_end_tokens=cooldown_end_tokens,
                   context_fork=context_fork, batch_tokens=batch_tokens, lr_scale=lr_scale)
    cfg = req.cfg
    batch_change = req.branch.record() if req.branch is not None else None
    if cfg.raw.get("project", {}).get("dry_run", True):
        return {**plan_search(cfg), "batch_branch": batch_change, "context_fork": context_fork,
                "new_context": cfg.raw.get("data", {}).get("context", 512),
                "parent": str(resume) if resume is not None else None,
                "parent_validation": "pending" if resume is not None else None}
    run_dir = Path(run_dir)
    dev, rate = _check_launch(req, run_dir, max_steps, max_seconds, device)
    project = cfg.raw.get("project", {})
    if _throughput_canary is not None:
        _throughput_canary.bind_output(run_dir / "canary.json")
    if resume is None:
        require_checkpoint_space(run_dir.parent, checkpoint_storage_plan(cfg, max_steps=max_steps)["required_additional_bytes"])
    first_context = _first_context(req)
    ledger = _ledger_for(project)
    run_id = str(run_dir.resolve())
    ledger.begin(run_id, rate, max_seconds, run_budget_usd, parent_checkpoint=resume,
                 cost_margin_fraction=project.get("cost_margin_fraction", .1), stage=project.get("stage", "A"))
    started = time.monotonic()
    status = "failed"
    try:
        run = _Run(req, run_dir, dev, rate, started=started, max_steps=max_steps, max_seconds=max_seconds,
                   first_context=first_context, ledger=ledger, run_id=run_id, profiler=_step_profiler,
                   canary=_throughput_canary)
        result = run.execute(batch_change)
        status = "complete"
        return result
    finally:
        try:
            if _step_profiler is not None:
                _step_profiler.close()
        finally:
            ledger.finish(run_id, time.monotonic() - started, status)


def _check_tokenizer(tokenizer: dict, named, dev):
    """The manifest's tokenizer must be the configured one (by name or fingerprint); test-only
    tokenizers (fixtures without a fingerprint) train on the CPU only."""
    if tokenizer.get("test_only") and dev.type != "cpu":
        raise ValueError("test-only tokenizer manifests are restricted to CPU fixtures")
    if named is not None and named not in (tokenizer["name"], tokenizer.get("fingerprint_sha256")):
        raise ValueError("configured tokenizer does not match immutable manifest")


def _assert_no_analysis_state(model):
    for name, module in model.named_modules():
        if getattr(module, "ablate", frozenset()):
            raise RuntimeError(f"analysis ablation leaked into training: {name}")
        if any(getattr(module, f, None) is not None for f in ("denom_mode", "denom_saved", "denom_const")):
            raise RuntimeError(f"analysis denominator state leaked into training: {name}")


@dataclass
class _Update:
    """What one optimizer update produced."""
    scheduler_step: int
    valid: int
    loss_sum: float
    anchor_sum: float
    grad_norm: torch.Tensor
    score_bound: float | None


class _Run:
    """One launched run: model, engine, sampler, lifecycles and the update loop."""

    def __init__(self, req: RunRequest, run_dir: Path, dev, rate, *, started, max_steps, max_seconds, first_context,
                 ledger, run_id, profiler, canary):
        self.req, self.cfg, self.run_dir, self.dev, self.rate = req, req.cfg, run_dir, dev, rate
        self.started, self.max_steps, self.max_seconds = started, max_steps, max_seconds
        self.first_context, self.ledger, self.run_id = first_context, ledger, run_id
        self.profiler, self.canary = profiler, canary
        self.region = getattr(profiler, "region", lambda _name: nullcontext())
        self.project, self.data = self.cfg.raw.get("project", {}), self.cfg.raw.get("data", {})
        self.parent = None

    # ------------------------------------------------------------------ set-up
    def _open_data(self):
        from .data import PackedSampler, manifest_hash
        self.sampler = PackedSampler(self.data["manifest"], split="train",
                                     batch_size=self.data.get("micro_batch_size", 1), context=self.first_context,
                                     seed=self.cfg.train.seed)
        self.manifest_hash = manifest_hash(self.data["manifest"])
        self.tokenizer = self.sampler.manifest["tokenizer"]
        _check_tokenizer(self.tokenizer, self.data.get("tokenizer"), self.dev)

    def _build_model(self):
        seed_all(self.cfg.train.seed)
        if self.dev.type == "cuda":
            torch.cuda.reset_peak_memory_stats(self.dev)
        self.model = TensorLM(self.cfg.model).to(self.dev)
        _assert_no_analysis_state(self.model)
        self.engine = TrainEngine(self.cfg, device=self.dev, model=self.model,
                                  optimizer=lambda m: make_optimizer(m, self.cfg.train))
        self.optimizer = self.engine.optimizer
        self.progress = {"steps": 0, "tokens": 0, "skipped_updates": [], "scheduler_step": 0, "input_tokens_seen": 0,
                         "discarded_prediction_targets": 0,
                         "warmup_steps": validate_schedule(self.cfg.train.schedule, self.req.planned_total)}

    def _load_parent(self) -> dict:
        """Load the parent checkpoint, apply a batch branch or context fork; returns its extras."""
        from .checkpoint import load_checkpoint
        req, progress, resume = self.req, self.progress, self.req.resume
        payload = load_checkpoint(resume, self.model, self.optimizer, self.sampler,
                                  expected_manifest_hash=self.manifest_hash, config_validator=req.validator,
                                  map_location="cpu")
        progress.update(payload["progress"])
        if payload.get("config_compatibility", {}).get("defaulted_fields"):
            progress.setdefault("config_compatibility_history", []).append(
                {"checkpoint": str(Path(resume).resolve()), **payload["config_compatibility"]})
        self.parent = {"path": str(Path(resume).resolve()),
                       "manifest_sha256": hashlib.sha256((Path(resume) / "manifest.json").read_bytes()).hexdigest()}
        if req.branch is not None:
            import yaml
            req.branch.check_parent(payload, self.cfg)
            req.branch.apply(self.optimizer, self.sampler, progress, req.parent_cfg, self.cfg, self.parent)
            (self.run_dir / "branch-config.yaml").write_text(yaml.safe_dump(full_config(self.cfg), sort_keys=False))
        if req.context_fork:
            from .runtime import record_context_fork
            before = self.sampler.state_dict()
            self.sampler = self.sampler.fork_context(self.data.get("context", 512))
            record_context_fork(progress, old_context=self.first_context, new_context=self.data.get("context", 512),
                                parent=self.parent, source_state=before)
        extra = payload.get("extra", {}) or {}
        if extra.get("cooldown_steps") is not None and not req.cooling:
            raise ValueError("cooldown checkpoint requires explicit matching cooldown_steps")
        return extra

    def _start_state(self):
        """Fresh progress or the parent's; then the cooldown's base rates and start."""
        req, progress = self.req, self.progress
        if req.resume:
            extra = self._load_parent()
        else:
            extra = {}
            progress["batch_history"] = [segment(self.cfg, tokens=0, steps=0, source="fresh")]
            progress["context_history"] = [{"context": self.data.get("context", 512), "start_tokens": 0,
                                            "start_step": 0, "source": "fresh"}]
        self.branch_base_lr = [g["lr"] for g in self.optimizer.param_groups]
        if not req.cooling:
            return
        if extra.get("cooldown_steps") is not None:
            if extra["cooldown_steps"] != req.cooldown_steps:
                raise ValueError("cannot change an existing cooldown horizon")
            if req.cooldown_end_tokens != extra.get("cooldown_end_tokens"):
                raise ValueError("cannot change an existing cooldown endpoint")
            self.branch_base_lr = extra["branch_base_lr"]
        else:
            progress["scheduler_step"] = 0
            progress["cooldown_start_tokens"] = progress["tokens"]

    def _token_limit(self) -> int:
        cfg, progress, req = self.cfg, self.progress, self.req
        if not req.cooling:
            return cfg.train.rung_total_tokens
        per_update = cfg.train.global_prediction_tokens_per_update
        limit = progress["cooldown_start_tokens"] + req.cooldown_steps * per_update
        end = req.cooldown_end_tokens
        if end is None:
            return limit
        if not limit - per_update < end <= limit:
            raise ValueError("cooldown endpoint must match the cooldown step horizon")
        progress["cooldown_end_tokens"] = end
        return end

    def _save(self, name) -> Path:
        from .checkpoint import save_checkpoint
        req, dev = self.req, self.dev
        save_checkpoint(self.run_dir / name, self.model, self.optimizer, self.sampler, config=full_config(self.cfg),
                        progress=self.progress, manifest_hash=self.manifest_hash, parent=self.parent,
                        extra={"operator_audit": self.model.operator_audit(), "cooldown_steps": req.cooldown_steps,
                               "cooldown_end_tokens": req.cooldown_end_tokens, "branch_base_lr": self.branch_base_lr,
                               "runtime": {"determinism": determinism_metadata(), "device": str(dev),
                                           "fused_sm100a_path": self.model.uses_fused_path(torch.empty(1, device=dev)),
                                           "autocast_enabled": False,
                                           "compute_dtype": "bfloat16" if dev.type == "cuda" else "float32"}})
        return self.run_dir / name

    # ------------------------------------------------------------------ one update
    def _set_rates(self) -> int:
        req, progress = self.req, self.progress
        sched = progress.get("scheduler_step", progress["steps"])
        if req.cooling:
            mult = lr_multiplier(sched, req.planned_total, cooldown_steps=req.cooldown_steps)
        else:
            mult = schedule_multiplier(sched, req.planned_total, schedule=self.cfg.train.schedule,
                                       warmup_steps=progress["warmup_steps"])
        for group, base in zip(self.optimizer.param_groups, self.branch_base_lr):
            group["lr"] = (base if req.cooling else group.get("base_lr", self.cfg.train.lr)) * mult
        return sched

    def _micro_batch(self, idx, docs, targets, n):
        """Forward and backward of one micro-batch with the norms' statistics collection; returns
        (summed loss, anchor penalty × targets)."""
        taper, lagged = self.taper, self.lagged
        with self.region("tnlm.transfer"):
            idx, docs, targets = (t.to(self.dev, non_blocking=True) for t in (idx, docs, targets))
        if taper.enabled:
            taper.set_valid_mask((docs >= 0) if taper.collecting else (targets != -100))
        for norm in lagged:
            norm.collecting = True
            norm.set_valid_mask(docs >= 0)
        try:
            with self.region("tnlm.forward"):
                loss, counted = self.engine.forward_loss(idx, docs, targets)
            if self.bounds.enabled:
                self.bounds.observe()
            anchor = taper.anchor()
            objective = loss if anchor is None else loss + taper.anchor_lambda * anchor * n
            with self.region("tnlm.validate_loss"):
                if int(counted) != n or not torch.isfinite(objective):
                    raise FloatingPointError("invalid loss/count; update aborted")
            with self.region("tnlm.backward"):
                self.engine.backward(objective)
        finally:
            taper.set_valid_mask(None)
            for norm in lagged:
                norm.collecting = False
                norm.set_valid_mask(None)
        return loss, (float(anchor.detach()) * n if anchor is not None else 0.0)

    def _update(self, token_limit) -> _Update:
        progress = self.progress
        self.bounds.begin_update()
        self.taper.before_step(progress["steps"])
        sched = self._set_rates()
        self.engine.begin_update()
        with self.region("tnlm.spectral_step"):
            spectral_step(self.model)
        wanted = min(self.cfg.train.global_prediction_tokens_per_update, token_limit - progress["tokens"])
        valid, loss_sum, anchor_sum = 0, 0.0, 0.0
        for idx, docs, targets, n in self.batcher.micro_batches(wanted, self.started + self.max_seconds):
            loss, anchor = self._micro_batch(idx, docs, targets, n)
            valid += n
            anchor_sum += anchor
            with self.region("tnlm.loss_accounting"):
                loss_sum += float(loss.detach())
        bound = self.bounds.finish_update() if self.bounds.enabled else None
        with self.region("tnlm.optimizer"):
            grad_norm = self.engine.finish_update(divide_by=valid, error_if_nonfinite=True)
        update_optimizer_exposure(progress, self.optimizer)
        for norm in self.lagged:
            norm.commit()
            _check_lagged_divisor(norm)
        if self.dev.type == "cuda":
            with self.region("tnlm.synchronize"):
                torch.cuda.synchronize(self.dev)
        progress["steps"] += 1
        self.taper.after_step(progress["steps"])
        progress["tokens"] += valid
        progress["scheduler_step"] = sched + 1
        return _Update(sched, valid, loss_sum, anchor_sum, grad_norm, bound)

    def _interventions(self):
        """QK-clip and the stability probe at their cadences: (clip report, probe report)."""
        policy, steps = self.req.policy, self.progress["steps"]
        clipping = stability = None
        if policy.clipping and steps % policy.clip_every == 0:
            with self.region("tnlm.qk_clip"):
                clipping = (self.bounds.clip(policy.clip_tau) if policy.clip_source == "batch_bound"
                            else self.probe.clip(self.model, policy.clip_tau))
        if policy.stability_every and steps % policy.stability_every == 0:
            with self.region("tnlm.stability_probe"):
                stability = self.probe.sample(self.model)
        return clipping, stability

    def _record(self, u: _Update, step_start, log: MetricsLog, clipping, stability) -> dict:
        progress, opt, batcher = self.progress, self.optimizer, self.batcher
        now = time.monotonic()
        record = {"step": progress["steps"], "tokens": progress["tokens"], "prediction_tokens": u.valid,
                  "loss": u.loss_sum / u.valid, "grad_norm": float(u.grad_norm),
                  "optimizer_group_lrs": [g["lr"] for g in opt.param_groups],
                  "optimizer_exposure": progress["optimizer_exposure"], "lr": opt.param_groups[0]["lr"],
                  "batch_hashes": batcher.hashes, "microbatches": len(batcher.hashes),
                  "forward_input_positions": batcher.positions, "unscored_rows_omitted": batcher.omitted,
                  "seconds": now - step_start}
        log.stamp(record, now)
        record.update(self.taper.metrics(u.anchor_sum / u.valid))
        for key, value in (("score_bound_max", u.score_bound), ("qk_clip", clipping), ("stability", stability)):
            if value is not None:
                record[key] = value
        return record

    # ------------------------------------------------------------------ the run
    def _prepare(self):
        """Everything between opening the data and the first update; returns (token limit, storage
        plan, disk admission, checkpoint schedule)."""
        cfg = self.cfg
        self._open_data()
        self.run_dir.mkdir(parents=True)
        self._build_model()
        self._start_state()
        progress = self.progress
        self.lagged = lagged_modules(self.model)
        if self.lagged and not self.req.resume:
            progress["calibration"] = calibrate_lagged(self.model, cfg, self.data["manifest"], self.dev,
                                                       deadline=self.started + self.max_seconds)
        for norm in self.lagged:
            _check_lagged_divisor(norm)
        self.bounds = BatchScoreBounds(self.model, cfg)
        token_limit = self._token_limit()
        plan = checkpoint_storage_plan(cfg, start_tokens=progress["tokens"], token_limit=token_limit,
                                       max_steps=self.max_steps, cooldown=self.req.cooling)
        admission = require_checkpoint_space(self.run_dir, plan["required_additional_bytes"])
        (self.run_dir / "checkpoint_storage_plan.json").write_text(
            json.dumps({"plan": plan, "admission": admission}, indent=2, allow_nan=False) + "\n")
        self.taper = TaperLifecycle(self.model, cfg, total_steps=self.req.planned_total,
                                    warmup_steps=progress["warmup_steps"])
        self.taper.before_step(progress["steps"])
        self.taper.set_valid_mask(None)
        milestones = pending_milestone_tokens(cfg, start_tokens=progress["tokens"], token_limit=token_limit,
                                              reachable_tokens=plan["reachable_tokens"],
                                              include_branch=not self.req.cooling and cfg.train.schedule != "cosine")
        saves = CheckpointSchedule(self._save, retention=checkpoint_retention_policy(cfg), milestones=milestones,
                                   every_steps=int(self.project.get("checkpoint_every_steps", 0)),
                                   every_seconds=float(self.project.get("checkpoint_every_seconds", 300)),
                                   ledger=self.ledger)
        saves.initial()
        self.probe = TrainingStabilityProbe(cfg, self.dev) if self.req.policy.needs_probe() else None
        self.batcher = QuotaBatcher(self.sampler, cfg.model.vocab_size, progress,
                                    trim_rows=not self.lagged and not self.taper.enabled, region=self.region)
        return token_limit, plan, admission, saves

    def execute(self, batch_change) -> dict:
        token_limit, plan, admission, saves = self._prepare()
        progress = self.progress
        log = MetricsLog(self.run_dir / "metrics.jsonl", int(self.project.get("history_limit", 1000)), self.started,
                         self.rate, progress["tokens"])
        self.model.train()
        slowest, updates, warm_updates = 0.0, 0, 0
        stop_reason = "max_steps"
        for local_step in range(self.max_steps):
            _assert_no_analysis_state(self.model)
            elapsed = time.monotonic() - self.started
            if elapsed >= self.max_seconds or elapsed + slowest + saves.seconds_per_save >= self.max_seconds:
                stop_reason = "runtime_cap"
                break
            if progress["tokens"] >= token_limit:
                stop_reason = "token_limit"
                break
            step_start = time.monotonic()
            if self.profiler is not None:
                self.profiler.start_step(local_step)
            u = self._update(token_limit)
            updates += 1
            warm_updates += int(not self.req.cooling and u.scheduler_step < progress["warmup_steps"])
            record = self._record(u, step_start, log, *self._interventions())
            if self.profiler is not None:
                self.profiler.finish_step()
            slowest = max(slowest, time.monotonic() - step_start)
            log.append(record)
            if self.canary is not None:
                self.canary.observe(record)
            saves.after_update(progress)
        if self.canary is not None:
            self.canary.require_complete()
        final = self._save("final")
        return self._result(batch_change, final, plan, admission, log, stop_reason, updates, warm_updates)

    def _result(self, batch_change, final, plan, admission, log, stop_reason, updates, warm_updates) -> dict:
        from .evaluate import _training_descriptor
        cfg, dev, progress, req = self.cfg, self.dev, self.progress, self.req
        frozen = full_config(cfg)
        descriptor = _training_descriptor({"config": frozen, "progress": progress,
                                           "extra": {"cooldown_steps": req.cooldown_steps,
                                                     "cooldown_end_tokens": req.cooldown_end_tokens}})
        cuda = dev.type == "cuda"
        result = {"training_descriptor": descriptor, "batch_branch": batch_change, "checkpoint": str(final),
                  "checkpoint_storage_plan": plan, "checkpoint_storage_admission": admission,
                  "progress": progress, "history": list(log.history), "metrics_path": str(log.path),
                  "spend_ledger": str(self.ledger.path.resolve()), "run_id": self.run_id, "parent": self.parent,
                  "history_limit": log.history.maxlen,
                  "cuda_peak_allocated_bytes": torch.cuda.max_memory_allocated(dev) if cuda else None,
                  "cuda_peak_reserved_bytes": torch.cuda.max_memory_reserved(dev) if cuda else None,
                  "operator_audit": self.model.operator_audit(), "parameters": self.model.param_counts(),
                  "runtime": {"determinism": determinism_metadata(), "device": str(dev), "torch": str(torch.__version__),
                              "bf16_compute": cfg.train.bf16_compute and cuda},
                  "model_config": frozen["model"], "train_config": frozen["train"],
                  "data": {"manifest_sha256": self.manifest_hash, "context": self.data.get("context", 512),
                           "tokenizer": self.tokenizer},
                  "stop_reason": stop_reason, "compile_enabled": False, "warmup_steps": progress["warmup_steps"],
                  "warmup_fraction_of_completed_updates": warm_updates / updates if updates else None,
                  "warmup_dominates_completed_segment": warm_updates > .1 * updates,
                  "lagged_collection_policy": "all nonpadding tokens; once per optimizer step",
                  "elapsed_seconds_before_final_accounting": time.monotonic() - self.started}
        if self.canary is not None:
            result["throughput_canary"] = self.canary.report()
        if self.profiler is not None:
            result["kernel_profile"] = self.profiler.report()
        (self.run_dir / "result.json").write_text(json.dumps(result, indent=2))
        return result


# ====================================================================================== profiling
_TIMED_FIELDS = ("seconds", "prediction_tokens", "microbatches", "forward_input_positions", "unscored_rows_omitted")


def profile_run(cfg, run_dir, *, steps, warmup_steps=2, max_seconds, device="cuda", run_budget_usd=None,
                kernels=False, trace_steps=0) -> dict:
    """Time complete training steps (the declared warm-up excluded), optionally with kernel
    profiles and Chrome traces; writes ``profile.json`` into the run directory."""
    if isinstance(cfg, (str, Path)):
        cfg = Config.from_yaml(str(cfg))
    if steps <= 0 or warmup_steps < 0:
        raise ValueError("positive timed steps and nonnegative warmup_steps required")
    if type(trace_steps) is not int or not 0 <= trace_steps <= 100:
        raise ValueError("trace_steps must be an integer in [0, 100]")
    cuda = torch.device(device).type == "cuda"
    if kernels and not cuda:
        raise ValueError("kernel profiling requires a CUDA device")
    from .profiling import KernelProfile
    profiler = (KernelProfile(warmup_steps, trace_dir=Path(run_dir) / "traces", trace_steps=max(1, trace_steps),
                              cuda=cuda, kernels=kernels) if kernels or trace_steps else None)
    result = train_run(cfg, run_dir, max_steps=steps + warmup_steps, max_seconds=max_seconds, device=device,
                       run_budget_usd=run_budget_usd, **({"_step_profiler": profiler} if profiler else {}))
    if result.get("dry_run"):
        return {**result, "command": "profile", "warmup_steps": warmup_steps, "timed_steps": steps,
                "kernels": kernels, "trace_steps": trace_steps}
    metrics = Path(result["metrics_path"])
    rows = [json.loads(line) for line in metrics.read_text().splitlines()] if metrics.exists() else []
    timed_rows = rows[warmup_steps:]
    total = {key: sum(r[key] for r in timed_rows) for key in _TIMED_FIELDS}
    timed, seconds, tokens = len(timed_rows), total["seconds"], total["prediction_tokens"]
    report = {"command": "profile", "device": str(device), "determinism": result.get("runtime", {}).get("determinism"),
              "kernels": kernels, "trace_steps": trace_steps, "requested_timed_steps": steps,
              "completed_timed_steps": timed, "warmup_steps": warmup_steps, "completed_total_steps": len(rows),
              "timed_training_seconds": seconds, "timed_prediction_tokens": tokens,
              "timed_microbatches": total["microbatches"],
              "timed_forward_input_positions": total["forward_input_positions"],
              "timed_unscored_rows_omitted": total["unscored_rows_omitted"],
              "forward_positions_per_prediction_target": total["forward_input_positions"] / tokens if tokens else None,
              "mean_microbatches_per_step": total["microbatches"] / timed if timed else None,
              "prediction_tokens_per_second": tokens / seconds if seconds > 0 else None,
              "mean_training_step_seconds": seconds / timed if timed else None,
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
