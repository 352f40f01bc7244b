"""Batch-size / learning-rate branches of a serial run.

A branch resumes a full-state checkpoint taken after warm-up and continues it with a different
per-update target quota, every learning rate multiplied by one factor, and the optimizer moments,
step counters and schedule counters left as they are.  The rules match the reference's
(tnlm/batch_branch.py:6-76): a branch needs a checkpoint to start from, a constant-LR schedule
with no cooldown and no context fork, no TaperNorm (its gate schedule is frozen against the
parent's quota), a quota that actually changes, and a parent that finished warm-up and has not
reached the child's token horizon.

``BatchBranch`` holds one request.  ``BatchBranch.request`` checks the request against the
configuration and returns None when no branch was asked for; ``child_config`` derives the child's
configuration; ``check_parent`` vets the parent checkpoint's progress record; ``apply`` rescales
the live optimizer and appends the branch to the checkpoint's ``batch_history`` list (the segment
record that evaluation reads back; ``segment`` builds one).
"""
from __future__ import annotations

import copy
import math
from dataclasses import dataclass

SCALED_RATES = ("lr", "aux_adamw_lr")  # TrainConfig fields a branch multiplies


def _is_count(v) -> bool:
    return type(v) is int and v > 0


def _is_factor(v) -> bool:
    return type(v) in (int, float) and math.isfinite(v) and v > 0


def segment(cfg, *, tokens, steps, source) -> dict:
    """One ``batch_history`` record: the quota and rates in force from (tokens, steps) on."""
    return {"batch_tokens": cfg.train.global_prediction_tokens_per_update, "lr": cfg.train.lr,
            "aux_adamw_lr": cfg.train.aux_adamw_lr, "start_tokens": tokens, "start_step": steps,
            "source": source}


@dataclass(frozen=True)
class BatchBranch:
    old_batch_tokens: int
    new_batch_tokens: int
    lr_scale: float

    # ------------------------------------------------------------------ request
    @classmethod
    def request(cls, cfg, *, batch_tokens, lr_scale, resume, context_fork, cooldown_steps) -> "BatchBranch | None":
        if batch_tokens is None and lr_scale is None:
            return None
        train = cfg.train
        rules = (
            (lambda: resume is not None and batch_tokens is not None and lr_scale is not None,
             "a batch branch takes a checkpoint to resume, a new batch token quota and an LR scale, all three"),
            (lambda: _is_count(batch_tokens), "the branch batch token quota must be a positive integer"),
            (lambda: _is_factor(lr_scale), "the branch LR scale must be a finite positive number"),
            (lambda: not context_fork and cooldown_steps is None
             and train.schedule == "constant_with_separate_cooldown",
             "a batch branch continues a constant-LR schedule: no cooldown and no context fork"),
            (lambda: "taper" not in (cfg.model.normalization, cfg.model.final_normalization),
             "a batch branch of a TaperNorm model would move its frozen gate schedule"),
            (lambda: batch_tokens != train.global_prediction_tokens_per_update,
             "a batch branch must change the batch token quota"),
        )
        for holds, message in rules:
            if not holds():
                raise ValueError(message)
        return cls(train.global_prediction_tokens_per_update, batch_tokens, float(lr_scale))

    def record(self) -> dict:
        return {"old_batch_tokens": self.old_batch_tokens, "new_batch_tokens": self.new_batch_tokens,
                "lr_scale": self.lr_scale}

    # ------------------------------------------------------------------ configuration and parent
    def child_config(self, cfg):
        child = copy.deepcopy(cfg)
        child.train.global_prediction_tokens_per_update = self.new_batch_tokens
        for name in SCALED_RATES:
            rate = getattr(child.train, name)
            if rate is None:
                continue
            if not _is_factor(rate * self.lr_scale):
                raise ValueError(f"the branch's scaled {name} is not a finite positive number")
            setattr(child.train, name, rate * self.lr_scale)
        return child

    @staticmethod
    def check_parent(payload, child_cfg) -> None:
        progress = payload["progress"]
        extra = payload.get("extra", {})
        cooling = (extra.get("cooldown_steps") is not None or "cooldown_start_tokens" in progress
                   or progress.get("distributed_schedule", {}).get("cooldown_steps") is not None)
        if cooling:
            raise ValueError("a batch branch cannot start from a cooldown checkpoint")
        warmup, sched = progress.get("warmup_steps"), progress.get("scheduler_step")
        if not (_is_count(warmup) and type(sched) is int and sched >= warmup):
            raise ValueError("a batch branch starts after the parent's warm-up, with its scheduler state recorded")
        tokens, steps = progress.get("tokens"), progress.get("steps")
        if not (type(tokens) is int and type(steps) is int and tokens >= 0 and steps >= 0):
            raise ValueError("the parent checkpoint's cumulative tokens and steps are missing or invalid")
        if tokens >= child_cfg.train.rung_total_tokens:
            raise ValueError("the parent has already reached the branch's token horizon")

    # ------------------------------------------------------------------ live state
    def apply(self, optimizer, sampler, progress, parent_cfg, child_cfg, parent) -> None:
        """Scale every group's ``lr`` and ``base_lr`` (all checked before any is changed) and
        append this branch to ``progress['batch_history']``."""
        def groups_view():
            return [{k: copy.deepcopy(v) for k, v in g.items() if k != "params"} for g in optimizer.param_groups]

        before = groups_view()
        new_rates = []
        for g in optimizer.param_groups:
            rates = {"lr": float(g["lr"]) * self.lr_scale, "base_lr": float(g.get("base_lr", g["lr"])) * self.lr_scale}
            if not all(_is_factor(v) for v in rates.values()):
                raise ValueError("a scaled optimizer group rate is not a finite positive number")
            new_rates.append(rates)
        for g, rates in zip(optimizer.param_groups, new_rates):
            g.update(rates)
        history = progress.setdefault("batch_history",
                                      [segment(parent_cfg, tokens=None, steps=None, source="legacy_unknown")])
        entry = segment(child_cfg, tokens=progress["tokens"], steps=progress["steps"], source="batch_branch")
        entry.update(lr_scale=self.lr_scale, parent=copy.deepcopy(parent),
                     source_sampler=copy.deepcopy(sampler.state_dict()),
                     optimizer_groups_before=before, optimizer_groups_after=groups_view(),
                     optimizer_policy="every group's lr and base_lr scaled; moments, step counts, betas, "
                                      "momentum and weight decay kept",
                     schedule_policy="warm-up and scheduler counters kept from the parent; constant LR continues")
        history.append(entry)
