"""Throughput canary: a pass/fail gate on the first completed training updates after warm-up.

The trainer reports each completed global update (step number, prediction targets scored, device
seconds).  Updates up to ``warmup_steps`` are ignored; the next ``measured_steps`` are collected and
the gate passes when their summed targets over their summed seconds reach ``min_tokens_per_second``.
The canary is a state machine::

    pending --first measured update--> collecting --last one--> passed | below_threshold
    (any state but passed) --require_complete()--> insufficient

``below_threshold`` raises at once so a slow run stops early; ``insufficient`` is raised when the
run ends before the gate decided.  Each transition is published to ``output_path`` (a durable JSON
file that must not exist when bound).  A pass says nothing about completing the run, later
throughput or model quality, and observing never touches tensors, optimizer, sampler or RNG.
Same gate and report schema as the reference (tnlm/throughput_canary.py:11-118).
"""
from __future__ import annotations

import math
from pathlib import Path

from .durable import write_json

PENDING, COLLECTING, PASSED, BELOW, INSUFFICIENT = "pending", "collecting", "passed", "below_threshold", "insufficient"


class ThroughputCanary:
    def __init__(self, measured_steps, min_tokens_per_second, warmup_steps, *, output_path=None):
        if type(measured_steps) is not int or measured_steps < 1:
            raise ValueError("measured_steps must be a positive integer")
        if type(warmup_steps) is not int or warmup_steps < 0:
            raise ValueError("warmup_steps must be a nonnegative integer")
        rate = min_tokens_per_second
        if type(rate) not in (int, float) or not math.isfinite(rate) or rate <= 0:
            raise ValueError("min_tokens_per_second must be a finite positive number")
        self.measured_steps = measured_steps
        self.warmup_steps = warmup_steps
        self.min_tokens_per_second = float(rate)
        self.output_path: Path | None = None
        self.records: list[dict] = []
        self.status = PENDING
        self.last_step = 0
        if output_path is not None:
            self.bind_output(output_path)

    @property
    def required_updates(self) -> int:
        return self.warmup_steps + self.measured_steps

    def bind_output(self, path) -> None:
        """Choose where reports go (once; rebinding to the same path is a no-op)."""
        path = Path(path)
        if self.output_path is not None:
            if path.absolute() != self.output_path.absolute():
                raise ValueError("the canary already publishes to another path")
            return
        if path.exists() or path.is_symlink():
            raise FileExistsError(path)
        self.output_path = path

    def _rate(self):
        seconds = sum(r["seconds"] for r in self.records)
        return sum(r["prediction_tokens"] for r in self.records) / seconds if seconds else None

    def report(self) -> dict:
        return {"kind": "throughput_canary", "status": self.status,
                "controls": {"measured_steps": self.measured_steps, "warmup_steps": self.warmup_steps,
                             "min_tokens_per_second": self.min_tokens_per_second},
                "selected_steps": list(self.records), "completed_measured_steps": len(self.records),
                "prediction_tokens": sum(r["prediction_tokens"] for r in self.records),
                "training_seconds": sum(r["seconds"] for r in self.records), "tokens_per_second": self._rate(),
                "timing_scope": "summed prediction targets over summed seconds of completed updates (micro-batch "
                                "accumulation, forward, backward and optimizer step; checkpoint writes excluded)",
                "scope": "a throughput gate only: passing implies nothing about finishing the run, later "
                         "throughput or model quality"}

    def _publish(self) -> None:
        if self.output_path is not None:
            self.output_path.parent.mkdir(parents=True, exist_ok=True)
            write_json(self.output_path, self.report())

    def observe(self, record: dict) -> None:
        """Take one completed update ``{"step", "prediction_tokens", "seconds"}``."""
        if self.status == PASSED:
            return
        if self.status in (BELOW, INSUFFICIENT):
            raise RuntimeError(f"the throughput canary has already failed ({self.status})")
        step = record.get("step")
        if type(step) is not int or step <= self.last_step:
            raise ValueError("canary steps must be positive integers that strictly increase")
        self.last_step = step
        if step <= self.warmup_steps:
            return
        tokens, seconds = record.get("prediction_tokens"), record.get("seconds")
        if type(tokens) is not int or tokens <= 0:
            raise ValueError("a measured update must score a positive number of targets")
        if type(seconds) not in (int, float) or not math.isfinite(seconds) or seconds <= 0:
            raise ValueError("a measured update must take a finite positive number of seconds")
        self.records.append({"step": step, "prediction_tokens": tokens, "seconds": float(seconds)})
        self.status = COLLECTING
        if len(self.records) == self.measured_steps:
            self.status = PASSED if self._rate() >= self.min_tokens_per_second else BELOW
        self._publish()
        if self.status == BELOW:
            raise RuntimeError(f"throughput {self._rate():.1f} tokens/s is below the canary's "
                               f"{self.min_tokens_per_second:.1f}")

    def require_complete(self) -> dict:
        if self.status != PASSED:
            self.status = INSUFFICIENT
            self._publish()
            raise RuntimeError("the run ended before the throughput canary measured all its updates")
        return self.report()
