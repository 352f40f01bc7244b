"""TaperNorm lifecycle in a training loop, driven by cumulative optimizer steps.

Phases, for a run of ``total_steps`` updates with ``warmup_steps`` of warm-up:

* warm-up (steps < warmup): the gate is 1 and every TaperRMS collects statistics over the tokens
  the trainer marks valid (non-padding); each completed update commits them (summed across ranks);
* taper (warmup <= step < end, end = round(taper_end_fraction * total_steps)): the norms are frozen
  (c, s_tgt and weight_tilde fixed from the warm-up statistics) and the shared cosine gate falls
  from 1 to 0; the trainer adds ``taper_anchor_lambda`` times the anchor term, weighted over the
  selected prediction targets like the cross-entropy;
* done (step >= end): gate 0, every norm is the fixed diagonal map.

A run resumed after warm-up freezes on its first step; a checkpoint whose norms are frozen cannot
resume inside warm-up.  The gate applied during a step is the one for the step number it started
from, and the gate stored at the end of a step is the next step's.  Same policy as the reference
(tnlm/training_taper.py:11-133).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from .models.normalization import taper_anchor_loss, taper_gate, taper_modules, taper_set_gate_

_EMA_FIELDS = ("ema_num", "ema_den", "ema_r", "ema_steps")


def is_taper_config(cfg) -> bool:
    return "taper" in (cfg.model.normalization, cfg.model.final_normalization)


@dataclass(frozen=True)
class TaperPolicy:
    anchor_lambda: float
    end_fraction: float
    ema_rate: float

    @classmethod
    def from_config(cls, cfg) -> "TaperPolicy | None":
        """The validated policy of a TaperNorm configuration; None when the model has no TaperNorm."""
        if not is_taper_config(cfg):
            return None

        def number(value, where):
            if type(value) not in (int, float) or not math.isfinite(value):
                raise ValueError(f"{where} must be a finite number")
            return float(value)
        policy = cls(number(cfg.train.taper_anchor_lambda, "train.taper_anchor_lambda"),
                     number(cfg.train.taper_end_fraction, "train.taper_end_fraction"),
                     number(cfg.model.taper_ema_rate, "model.taper_ema_rate"))
        if policy.anchor_lambda < 0:
            raise ValueError("train.taper_anchor_lambda must be nonnegative")
        if not 0 < policy.end_fraction <= 1:
            raise ValueError("train.taper_end_fraction must lie in (0, 1]")
        if not 0 < policy.ema_rate <= 1:
            raise ValueError("model.taper_ema_rate must lie in (0, 1]")
        if cfg.train.compile:
            raise ValueError("TaperNorm training needs train.compile: false (its statistics are Python-side)")
        if cfg.model.activation_checkpointing:
            raise ValueError("TaperNorm cannot use activation checkpointing (recomputed forwards would count twice)")
        return policy

    def end_step(self, total_steps: int) -> int:
        return round(self.end_fraction * total_steps)


def validate_taper_config(cfg) -> bool:
    """True for a valid TaperNorm configuration, False without TaperNorm; raises if invalid."""
    return TaperPolicy.from_config(cfg) is not None


class TaperLifecycle:
    def __init__(self, model, cfg, *, total_steps, warmup_steps, distributed=False):
        self.model = model
        self.policy = TaperPolicy.from_config(cfg)
        self.enabled = self.policy is not None
        self.norms = taper_modules(model) if self.enabled else []
        self.anchor_lambda = self.policy.anchor_lambda if self.enabled else 0.0
        self.distributed = distributed
        self.warmup_steps = warmup_steps
        self.end_step = total_steps
        self._step: int | None = None  # the update in progress
        self._gate_used = 1.0
        self._constants_reported = False
        if not self.enabled:
            return
        if type(total_steps) is not int or total_steps <= 0:
            raise ValueError("TaperNorm needs a positive integer number of total steps")
        self.end_step = self.policy.end_step(total_steps)
        if type(warmup_steps) is not int or warmup_steps <= 0 or self.end_step <= warmup_steps:
            raise ValueError("the TaperNorm end step must come strictly after a positive number of warm-up steps")
        if not self.norms:
            raise ValueError("the TaperNorm configuration built no TaperRMS modules")

    @property
    def collecting(self) -> bool:
        return self.enabled and self._step is not None and self._step < self.warmup_steps

    def _freeze_all(self):
        for norm in self.norms:
            norm.collecting = False
            norm.freeze()

    def _apply_gate(self, step: int) -> float:
        gate = taper_gate(step, self.warmup_steps, self.end_step)
        taper_set_gate_(self.model, gate)
        return gate

    def before_step(self, step: int) -> None:
        if not self.enabled:
            return
        if type(step) is not int or step < 0:
            raise ValueError("a TaperNorm step number is a nonnegative integer")
        self._step = step
        if step >= self.warmup_steps:
            self._freeze_all()
        elif any(bool(n.frozen) for n in self.norms):
            raise ValueError("a frozen TaperNorm cannot resume inside its warm-up")
        self._gate_used = self._apply_gate(step)
        for norm in self.norms:
            norm.collecting = self.collecting

    def set_valid_mask(self, mask) -> None:
        """Tokens the next forward counts (None: none, which also stops statistics collection, for
        probes and checkpoint boundaries)."""
        for norm in self.norms:
            norm.set_valid_mask(mask)
            norm.collecting = mask is not None and self.collecting

    def anchor(self):
        return taper_anchor_loss(self.model) if self.enabled else None

    def after_step(self, completed_steps: int) -> None:
        if not self.enabled:
            return
        if self._step is None or completed_steps != self._step + 1:
            raise ValueError("TaperNorm after_step must follow exactly one optimizer update")
        committing = self.collecting
        self.set_valid_mask(None)
        if committing:
            # every rank runs every module's collective before a local failure may surface
            for norm in self.norms:
                norm.commit(distributed=self.distributed)
            for norm in self.norms:
                if not all(bool(torch.isfinite(getattr(norm, f))) for f in _EMA_FIELDS):
                    raise FloatingPointError("a TaperNorm warm-up statistic became non-finite")
        if completed_steps >= self.warmup_steps:
            self._freeze_all()
        self._apply_gate(completed_steps)
        self._step = None

    def metrics(self, anchor_average) -> dict:
        if not self.enabled:
            return {}
        out = {"taper_gate": float(self.norms[0].gate), "taper_gate_used": self._gate_used,
               "taper_anchor": float(anchor_average)}
        if not self._constants_reported and all(bool(n.frozen) for n in self.norms):
            ids = {id(n) for n in self.norms}
            out["taper_constants"] = {name: {"c": float(m.c), "s_tgt": float(m.s_tgt)}
                                      for name, m in self.model.named_modules() if id(m) in ids}
            self._constants_reported = True
        return out
