"""Frozen held-out evaluation, paired comparisons and exact-label mechanism probes
(reference tnlm/evaluate.py:22-945).

* ``evaluate_checkpoint``: CE on a context-independent validation target plan (source target
  offsets 1..L-1 of documents in ``documents.jsonl`` order, up to a token cap), with a
  document-bootstrap CI, proof that the model/buffers were not mutated, and an exact-document
  overlap audit of the validation split against training data;
* ``compare_evaluations``: paired per-document bootstrap of CE_right - CE_left on identical plans;
* ``evaluate_mechanisms``: answer-token CE/accuracy on held-out task compositions, branch removal
  and final-position activation transfer between same-task donors;
* ``_training_descriptor`` / ``_training_comparison``: what a checkpoint says about its training.
"""
from __future__ import annotations

import copy
import hashlib
import json
import math
import os
import time
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

from .budget import SpendLedger
from .calibration import _check_lagged_divisor
from .config import Config
from .models.model import TensorLM
from .models.normalization import lagged_modules
from .hashing import canonical_sha256
from .runtime import evaluation_validator


def _integer(v, minimum=0):
    return v if type(v) is int and v >= minimum else None


def _number(v, nonnegative=True):
    return v if type(v) in (int, float) and math.isfinite(v) and (not nonnegative or v >= 0) else None


def _history(progress, key, check_entry, fresh_source, fork_source, last_check):
    history = progress.get(key)
    if not isinstance(history, list) or not history:
        return None, "unknown"
    entries, complete = [], True
    prev_tokens = prev_step = None
    for i, e in enumerate(history):
        if not isinstance(e, dict) or not check_entry(e, entries):
            return None, "unknown"
        tokens, step, source = e.get("start_tokens"), e.get("start_step"), e.get("source")
        if i == 0 and source == "legacy_unknown" and tokens is None and step is None:
            complete = False
        else:
            if any(type(v) is not int or v < 0 for v in (tokens, step)):
                return None, "unknown"
            if i == 0 and (source != fresh_source or tokens != 0 or step != 0):
                return None, "unknown"
            if i > 0 and (source != fork_source or (prev_tokens is not None and tokens < prev_tokens)
                          or (prev_step is not None and step < prev_step)):
                return None, "unknown"
            if (type(progress.get("tokens")) is not int or tokens > progress["tokens"]
                    or type(progress.get("steps")) is not int or step > progress["steps"]):
                return None, "unknown"
        entries.append(e)
        prev_tokens, prev_step = tokens, step
    if not last_check(entries[-1]):
        return None, "unknown"
    return entries, "complete" if complete else "partial"


def _context_history_descriptor(progress, context):
    def check(e, prior):
        ctx = e.get("context")
        return type(ctx) is int and ctx > 0 and (not prior or e.get("source") == "legacy_unknown"
                                                 or ctx > prior[-1]["context"])
    entries, status = _history(progress, "context_history", check, "fresh", "context_fork",
                               lambda last: last["context"] == context)
    if entries is None:
        return None, status
    return [{k: e.get(k) for k in ("context", "start_tokens", "start_step", "source")} for e in entries], status


def _batch_history_descriptor(progress, train):
    rate = lambda v: type(v) in (int, float) and math.isfinite(v) and v >= 0  # noqa: E731

    def check(e, prior):
        batch, scale = e.get("batch_tokens"), e.get("lr_scale", 1.0)
        ok = (type(batch) is int and batch > 0 and rate(e.get("lr")) and "aux_adamw_lr" in e
              and (e["aux_adamw_lr"] is None or rate(e["aux_adamw_lr"])) and rate(scale) and scale > 0)
        if not prior and scale != 1:
            return False
        if prior and e.get("source") == "batch_branch" and "lr_scale" not in e:
            return False
        return ok

    def last_ok(last):
        return (last["batch_tokens"] == train.get("global_prediction_tokens_per_update")
                and last["lr"] == train.get("lr") and last["aux_adamw_lr"] == train.get("aux_adamw_lr"))
    entries, status = _history(progress, "batch_history", check, "fresh", "batch_branch", last_ok)
    if entries is None:
        return None, status
    return [{"batch_tokens": e["batch_tokens"], "lr": e["lr"], "aux_adamw_lr": e["aux_adamw_lr"],
             "start_tokens": e.get("start_tokens"), "start_step": e.get("start_step"), "source": e.get("source"),
             "lr_scale": e.get("lr_scale", 1.0)} for e in entries], status


class _SegmentEvidence:
    """What a checkpoint payload says about the training segment it ends: whether the segment is a
    cooldown branch ("cooled", with its step horizon), a run on its own rung ("uncooled"), or
    undecidable; the segment's token endpoint; and whether the checkpoint reached it.  Every
    inconsistency leaves a note and turns the affected verdict to "unknown"; nothing missing is
    filled in.  The verdicts and note texts are the reference's report vocabulary (evaluation
    reports from either framework compare with each other)."""

    def __init__(self, progress: dict, extra: dict, train: dict):
        self.notes: list[str] = []
        self.tokens = _integer(progress.get("tokens"))
        self.rung = _integer(train.get("rung_total_tokens"), 1)
        self.batch = _integer(train.get("global_prediction_tokens_per_update"), 1)
        self.scheduler_step = _integer(progress.get("scheduler_step"))
        self.start = _integer(progress.get("cooldown_start_tokens"))
        self.status, self.steps = self._branch(progress.get("distributed_schedule"), extra)
        self.target, explicit_end_invalid = self._endpoint(progress)
        self.completion = self._reached(explicit_end_invalid, cosine=train.get("schedule") == "cosine")

    def _unknown(self, note: str, value=None):
        self.notes.append(note)
        return value

    def _branch(self, schedule, extra) -> tuple:
        """(status, cooldown steps) from the horizons the payload declares in its two places."""
        declared = set()
        for record in (schedule, extra):
            if isinstance(record, dict) and "cooldown_steps" in record:
                steps = record["cooldown_steps"]
                if steps is None or _integer(steps, 1) is not None:
                    declared.add(steps)
        if len(declared) > 1:
            return self._unknown("conflicting checkpoint cooldown metadata", ("unknown", None))
        if declared:
            steps = declared.pop()
            if steps is not None:
                return "cooled", steps
            if self.start is None:
                return "uncooled", None
            return self._unknown("cooldown start conflicts with explicit uncooled metadata", ("unknown", None))
        if self.start is not None:
            return self._unknown("cooldown branch start exists but its step horizon is missing", ("cooled", None))
        return self._unknown("checkpoint has no explicit cooldown branch evidence", ("unknown", None))

    def _endpoint(self, progress) -> tuple:
        """(token endpoint of the segment or None, whether an explicit endpoint was refused)."""
        horizon = None
        if self.status == "uncooled":
            horizon = self.rung
        elif self.status == "cooled" and None not in (self.start, self.steps, self.batch):
            horizon = self.start + self.steps * self.batch
        if "cooldown_end_tokens" not in progress:
            return horizon, False
        end = _integer(progress["cooldown_end_tokens"], 1)
        # an explicit endpoint lies inside the last update of the branch's horizon
        if (self.status == "cooled" and None not in (end, self.start, self.steps, self.batch)
                and self.start + (self.steps - 1) * self.batch < end <= self.start + self.steps * self.batch):
            return end, False
        return self._unknown("invalid explicit cooldown token endpoint", (None, True))

    def _reached(self, explicit_end_invalid: bool, *, cosine: bool) -> str:
        verdict = "unknown"
        if self.target is not None and self.tokens is not None:
            reached = self.tokens >= self.target
            verdict = "complete" if reached else "partial"
            if (self.status == "cooled" and self.scheduler_step is not None
                    and reached != (self.scheduler_step >= self.steps)):
                verdict = self._unknown("cooldown token and scheduler-step completion evidence disagree", "unknown")
        elif (not explicit_end_invalid and self.status == "cooled" and None not in (self.steps, self.scheduler_step)):
            verdict = "complete" if self.scheduler_step >= self.steps else "partial"
        if cosine and not self._cosine_consistent():
            verdict = self._unknown("cosine token and scheduler horizon evidence is missing or inconsistent",
                                    "unknown")
        return verdict

    def _cosine_consistent(self) -> bool:
        """A cosine run has no separate cooldown and reaches its rung exactly at its last update."""
        if self.status != "uncooled" or None in (self.rung, self.batch, self.scheduler_step, self.tokens):
            return False
        updates = -(-self.rung // self.batch)
        return (self.scheduler_step <= updates and self.tokens <= self.rung
                and (self.tokens == self.rung) == (self.scheduler_step == updates))


def _training_descriptor(payload) -> dict:
    """Training evidence recorded in a checkpoint payload (never evaluation overrides)."""
    def section(mapping, key):
        value = mapping.get(key) if isinstance(mapping, dict) else None
        return value if isinstance(value, dict) else {}
    config, progress, extra = (section(payload, k) for k in ("config", "progress", "extra"))
    train, model, data = (section(config, k) for k in ("train", "model", "data"))
    ctx_hist, ctx_status = _context_history_descriptor(progress, data.get("context", 512))
    batch_hist, batch_status = _batch_history_descriptor(progress, train)
    segment = _SegmentEvidence(progress, extra, train)

    def text(v):
        return v if isinstance(v, str) and v else None

    def positive_or_disabled(key):  # an explicit null switches the scaling rule off
        return "disabled" if key in model and model[key] is None else _integer(model.get(key), 1)
    descriptor = {
        "version": 1, "source": "checkpoint_payload",
        "config_compatibility": copy.deepcopy(payload.get("config_compatibility", {})),
        "configuration": copy.deepcopy({k: v for k, v in config.items() if k != "project"}),
        "optimizer": text(train.get("optimizer")), "seed": _integer(train.get("seed")),
        "width": _integer(model.get("d_model"), 1), "depth": _integer(model.get("layers"), 1),
        "train_context": _integer(data.get("context"), 1), "rung_total_tokens": segment.rung,
        "context_history": ctx_hist, "context_history_status": ctx_status,
        "batch_history": batch_hist, "batch_history_status": batch_status,
        "normalization": text(model.get("normalization")), "attention": text(model.get("attention")),
        "width_scaling_base": positive_or_disabled("width_scaling_base"),
        "depth_scaling_base": positive_or_disabled("depth_scaling_base"),
        "depth_residual_base": positive_or_disabled("depth_residual_base"),
    }
    for key in ("width_lr_exponent", "width_logit_exponent", "depth_lr_exponent", "depth_residual_exponent",
                "residual_alpha"):  # signed
        descriptor[key] = _number(model.get(key), False)
    for key in ("weight_decay_hidden", "beta1", "beta2", "lr"):
        descriptor[key] = _number(train.get(key))
    descriptor["aux_adamw_lr"] = ("default_to_lr" if "aux_adamw_lr" in train and train["aux_adamw_lr"] is None
                                  else _number(train.get("aux_adamw_lr")))
    descriptor.update({
        "actual_prediction_tokens": segment.tokens, "optimizer_steps": _integer(progress.get("steps")),
        "global_prediction_tokens_per_update": segment.batch, "schedule": text(train.get("schedule")),
        "scheduler_step": segment.scheduler_step, "warmup_steps": _integer(progress.get("warmup_steps"), 1),
        "cooldown_status": segment.status, "cooldown_steps": segment.steps,
        "cooldown_start_tokens": segment.start, "segment_target_prediction_tokens": segment.target,
        "completion_status": segment.completion, "evidence_notes": segment.notes,
        "completion_scope": "declared training segment token/step endpoint only; no automatic experiment "
                            "completion, fairness, or ranking claim"})
    return descriptor


_COMPARED = ("optimizer", "seed", "width", "depth", "train_context", "context_history", "batch_history",
             "rung_total_tokens", "actual_prediction_tokens", "global_prediction_tokens_per_update", "lr",
             "normalization", "attention", "width_scaling_base", "width_lr_exponent", "width_logit_exponent",
             "aux_adamw_lr", "schedule", "cooldown_status", "cooldown_steps", "segment_target_prediction_tokens",
             "completion_status", "warmup_steps", "depth_scaling_base", "depth_lr_exponent", "depth_residual_base",
             "depth_residual_exponent", "residual_alpha", "weight_decay_hidden", "beta1", "beta2")


def _comparable(report) -> dict:
    """The report's training descriptor, or {} when it is absent or of another version/source."""
    d = report.get("training_descriptor")
    return d if isinstance(d, dict) and d.get("version") == 1 and d.get("source") == "checkpoint_payload" else {}


def _dimension_value(d: dict, field: str):
    """A descriptor's value for one compared dimension: an uncooled run's absent cooldown horizon is
    "not_applicable" rather than missing, and a history counts only when it is complete."""
    value = d.get(field)
    if field == "cooldown_steps" and value is None and field in d and d.get("cooldown_status") == "uncooled":
        return "not_applicable"
    if field in ("context_history", "batch_history") and d.get(f"{field}_status") != "complete":
        return None
    return value


def _training_comparison(left, right) -> dict:
    """Per dimension: matched, different, or unknown when either side lacks the evidence (missing
    evidence is never taken as equal)."""
    sides = (_comparable(left), _comparable(right))
    dims, by_status = {}, {"matched": [], "different": [], "unknown": []}
    for field in _COMPARED:
        a, b = (_dimension_value(d, field) for d in sides)
        if any(v is None or v == "unknown" for v in (a, b)):
            status = "unknown"
        else:
            status = "matched" if a == b else "different"
        # the report shows the recorded values, also for a history that is not complete
        shown = [d.get(field) if field in ("context_history", "batch_history") else v
                 for d, v in zip(sides, (a, b))]
        dims[field] = {"status": status, "left": shown[0], "right": shown[1]}
        by_status[status].append(field)
    return {"dimensions": dims, "matched_dimensions": by_status["matched"],
            "different_dimensions": by_status["different"], "unknown_dimensions": by_status["unknown"],
            "automatic_ranking_eligible": False,
            "scope": "training evidence summary only; equality of missing evidence is never inferred"}


def _tensor_hash(items) -> str:
    """sha256 over (name, dtype, shape, raw bytes) of named tensors, in name order."""
    h = hashlib.sha256()
    for name, value in sorted(items):
        value = value.detach().cpu().contiguous()
        h.update(json.dumps([name, str(value.dtype), list(value.shape)]).encode())
        h.update(value.reshape(-1).view(torch.uint8).numpy().tobytes())
    return h.hexdigest()


def _file_hash(path, deadline=lambda: None) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as fh:
        for block in iter(lambda: fh.read(1 << 20), b""):
            deadline()
            h.update(block)
    return h.hexdigest()


def _ledger(project):
    return SpendLedger(project.get("spend_ledger", "runs/spend.json"), project.get("total_budget_usd", 1000),
                       project.get("reserve_usd", 150), stage_budgets=project.get("stage_budgets"))


def ratio_bootstrap(numerators, denominators, *, samples: int, seed: int):
    """95 % percentile interval of sum(numerators) / sum(denominators) under resampling of the
    units (documents) with replacement: ``samples`` resamples drawn one after another from
    ``numpy.random.default_rng(seed)``.  None with fewer than two units or no resamples."""
    num = np.asarray(numerators, dtype=np.float64)
    den = np.asarray(denominators, dtype=np.int64)
    units = len(num)
    if units < 2 or not samples:
        return None
    rng = np.random.default_rng(seed)
    ratios = np.empty(samples)
    for k in range(samples):
        pick = rng.integers(0, units, size=units)
        ratios[k] = num[pick].sum() / den[pick].sum()
    return np.quantile(ratios, [.025, .975]).tolist()


class TargetPlan:
    """The targets a held-out evaluation scores, independent of the probe context: for each
    validation document in the manifest's order, source target offsets 1 .. length-1 (every token
    that has a predecessor), until ``cap`` targets are planned.  The plan's canonical JSON digest
    is its identity: two evaluations are comparable only on the same plan."""

    def __init__(self, sampler, cap: int):
        self.ranges, left = [], cap
        for i in range(len(sampler.docs)):
            count = min(max(0, sampler.docs.length(i) - 1), left)
            if count:
                self.ranges.append({"document_id": sampler.docs[i]["id"], "target_start": 1,
                                    "target_end": count + 1, "count": count})
                left -= count
            if not left:
                break
        if not self.ranges:
            raise ValueError("validation split has no prediction targets")
        self.by_document = {r["document_id"]: r for r in self.ranges}
        self.record = {"version": 1, "validation_manifest_sha256": sampler.manifest_hash, "split": "val",
                       "ordering": "immutable documents.jsonl order",
                       "offset_semantics": "processed document stream; includes synthetic EOS if present",
                       "ranges": self.ranges}
        self.sha256 = canonical_sha256(self.record)

    def select(self, mappings, original, context):
        """Targets of one packed row restricted to the plan, and the chosen positions as
        (column, document id, available prefix length, source offset)."""
        targets = torch.full_like(original, -100)
        chosen = []
        for m in mappings:
            planned = self.by_document.get(m["document_id"])
            if planned is None:
                continue
            first, end = m["packed_token_start"], m["packed_token_end"]
            for col in range(first, min(end - 1, context)):
                offset = m["source_token_start"] + col - first + 1
                if not planned["target_start"] <= offset < planned["target_end"]:
                    continue
                if original[0, col] == -100:
                    raise ValueError("selected validation target was masked by sampler")
                targets[0, col] = original[0, col]
                chosen.append((col, m["document_id"], col - first + 1, offset))
        return targets, chosen


class _PlanScore:
    """Per-document loss sums of a target plan, checked to visit every planned offset exactly once
    and in order, with the histogram and digest of the prefixes the model saw."""

    def __init__(self, plan: TargetPlan):
        self.plan = plan
        self.totals = {r["document_id"]: {"loss_sum": 0.0, "tokens": 0} for r in plan.ranges}
        self.prefixes: dict[int, int] = {}
        self.prefix_digest = hashlib.sha256()
        self.forward_tokens = self.forward_batches = 0

    def add(self, losses, chosen, input_tokens):
        for col, doc, prefix, offset in chosen:
            total = self.totals[doc]
            if offset != self.plan.by_document[doc]["target_start"] + total["tokens"]:
                raise ValueError("duplicate or missing source target offset in evaluation")
            total["loss_sum"] += float(losses[col])
            total["tokens"] += 1
            self.prefixes[prefix] = self.prefixes.get(prefix, 0) + 1
            self.prefix_digest.update(json.dumps([doc, offset, prefix], separators=(",", ":")).encode() + b"\n")
        self.forward_batches += 1
        self.forward_tokens += input_tokens

    def finish(self):
        for r in self.plan.ranges:
            if self.totals[r["document_id"]]["tokens"] != r["count"]:
                raise ValueError("validation target plan was not evaluated exactly once")
        counts = [t["tokens"] for t in self.totals.values()]
        sums = [t["loss_sum"] for t in self.totals.values()]
        return counts, sums


def _frozen_state(model) -> tuple[str, str]:
    return _tensor_hash(model.state_dict().items()), _tensor_hash(model.named_buffers())


def _source_provenance(checkpoint_code) -> dict:
    pkg = Path(__file__).parent
    runtime_sources = {f"{pkg.name}/{p.relative_to(pkg).as_posix()}": _file_hash(p) for p in sorted(pkg.rglob("*.py"))}
    saved = checkpoint_code.get("source_sha256", {})
    critical = ("models/model.py", "models/attention.py", "models/normalization.py", "config.py")
    matches = {n: runtime_sources.get(f"{pkg.name}/{n}") == saved.get(f"{pkg.name}/{n}") for n in critical}
    return {"checkpoint_code": checkpoint_code, "runtime_source_sha256": runtime_sources,
            "critical_model_sources_match_checkpoint": all(matches.values()), "critical_model_source_matches": matches}


def _check_eval_bounds(context, max_prediction_tokens, bootstrap_samples, max_seconds):
    if (type(context) is not int or context <= 0 or type(max_prediction_tokens) is not int
            or max_prediction_tokens <= 0 or type(bootstrap_samples) is not int
            or not 0 <= bootstrap_samples <= 100_000 or not math.isfinite(max_seconds) or max_seconds <= 0):
        raise ValueError("positive evaluation bounds and bootstrap_samples in [0, 100000] required")


def _checked_rate(project, dev):
    if dev.type == "cuda" and not torch.cuda.is_available():
        raise RuntimeError("CUDA requested but unavailable")
    rate = project.get("gpu_hourly_rate_usd")
    if rate is None or (dev.type == "cuda" and rate <= 0):
        raise ValueError("declare actual gpu_hourly_rate_usd (explicit 0 allowed for CPU)")
    return rate


def _load_frozen_model(cfg, checkpoint, train_hash, dev):
    """The checkpoint's model in eval mode with its lagged statistics frozen; (model, payload)."""
    from .checkpoint import load_checkpoint
    model = TensorLM(cfg.model)
    payload = load_checkpoint(checkpoint, model, config_validator=evaluation_validator(cfg),
                              expected_manifest_hash=train_hash, restore_rng=False, map_location="cpu")
    model.to(dev).eval()
    for norm in lagged_modules(model):
        norm.collecting = False
        norm.set_valid_mask(None)
        _check_lagged_divisor(norm)
    return model, payload


def evaluate_checkpoint(cfg, checkpoint, out_dir, *, context=None, max_prediction_tokens=1_000_000, max_seconds,
                        device="cpu", bootstrap_samples=1000, run_budget_usd=None) -> dict:
    """Held-out CE of ``checkpoint`` on the validation target plan (see ``TargetPlan``), with a
    document-bootstrap interval, proof that evaluation left the model unchanged and an exact-document
    overlap audit against the training data; writes ``evaluation.json`` into ``out_dir``."""
    from .data import PackedSampler, audit_validation_overlap, manifest_hash, validate_tokenizer_compatibility
    if isinstance(cfg, (str, Path)):
        cfg = Config.from_yaml(str(cfg))
    project, data = cfg.raw.get("project", {}), cfg.raw.get("data", {})
    probe_context = data.get("context", 512) if context is None else context
    if project.get("dry_run", True):
        return {"dry_run": True, "command": "evaluate", "checkpoint": str(checkpoint), "context": probe_context,
                "max_prediction_tokens": max_prediction_tokens, "split": "val",
                "target_policy": "canonical document order; source target offsets 1..L-1"}
    _check_eval_bounds(probe_context, max_prediction_tokens, bootstrap_samples, max_seconds)
    dev = torch.device(device)
    rate = _checked_rate(project, dev)
    out_dir = Path(out_dir)
    if out_dir.exists():
        raise FileExistsError(f"evaluation directory already exists: {out_dir}")
    ledger = _ledger(project)
    run_id = str(out_dir.resolve())
    ledger.begin(run_id, rate, max_seconds, run_budget_usd, parent_checkpoint=checkpoint,
                 cost_margin_fraction=project.get("cost_margin_fraction", .1), stage=project.get("stage", "A"))
    started, status = time.monotonic(), "failed"

    def deadline():
        if time.monotonic() - started >= max_seconds:
            raise TimeoutError("evaluation runtime cap exhausted")

    try:
        out_dir.mkdir(parents=True, exist_ok=False)
        train_hash = manifest_hash(data["manifest"])
        evaluation = cfg.raw.get("evaluation", {})
        val_path = evaluation.get("validation_manifest", data["manifest"])
        tok_compat = validate_tokenizer_compatibility(data["manifest"], val_path, allow_test_only=dev.type == "cpu")
        eval_seed = int(evaluation.get("seed", 0))
        sampler = PackedSampler(val_path, split="val", batch_size=1, context=probe_context, seed=eval_seed)
        plan = TargetPlan(sampler, max_prediction_tokens)
        audit = audit_validation_overlap(data["manifest"], val_path, document_ids=[r["document_id"] for r in plan.ranges])
        (out_dir / "data-overlap-audit.json").write_text(json.dumps(audit, indent=2) + "\n")
        if audit["has_overlap"]:
            raise ValueError("held-out validation has exact whole-document content overlap; see data-overlap-audit.json")
        model, payload = _load_frozen_model(cfg, checkpoint, train_hash, dev)
        ckpt_progress, ckpt_code, descriptor = payload["progress"], payload["code"], _training_descriptor(payload)
        del payload
        before_model, before_buffers = _frozen_state(model)
        score = _PlanScore(plan)
        initial = sampler.state_dict()
        with torch.inference_mode():
            for _ in range(sampler.epoch_row_count):
                deadline()
                idx, docs, original = sampler.next_batch()
                targets, chosen = plan.select(sampler.batch_mappings()[0]["ranges"], original, probe_context)
                if not chosen:
                    continue
                logits = model(idx.to(dev), doc_ids=docs.to(dev))
                losses = F.cross_entropy(logits.float().flatten(0, 1), targets.to(dev).flatten(), reduction="none",
                                         ignore_index=-100).cpu()
                if not torch.isfinite(losses).all():
                    raise FloatingPointError("nonfinite validation loss")
                score.add(losses, chosen, int((docs >= 0).sum()))
        counts, sums = score.finish()
        after_model, after_buffers = _frozen_state(model)
        if (before_model, before_buffers) != (after_model, after_buffers):
            raise RuntimeError("evaluation changed checkpoint model or normalization buffers")
        tokens, loss_sum = int(np.sum(counts, dtype=np.int64)), float(np.sum(sums, dtype=np.float64))
        ci = ratio_bootstrap(sums, counts, samples=bootstrap_samples, seed=eval_seed)
        ckpt = Path(checkpoint)
        result = {"kind": "held_out_validation", "evaluation_protocol_version": 2, "data_overlap_audit": audit,
                  "tokenizer_compatibility": tok_compat, "split": "val", "context": probe_context,
                  "prediction_tokens": tokens, "loss_sum": loss_sum, "ce": loss_sum / tokens,
                  "validation_below_one_million_targets": tokens < 1_000_000,
                  "uncertainty": {"unit": "documents, not training seeds",
                                  "method": "token-weighted ratio document bootstrap", "samples": bootstrap_samples,
                                  "seed": eval_seed, "ce_95_ci": ci, "documents": len(score.totals)},
                  "target_plan": plan.record, "target_plan_sha256": plan.sha256,
                  "per_document": [{"document_id": k, **v} for k, v in score.totals.items()],
                  "available_prefix_length_histogram": {str(k): v for k, v in sorted(score.prefixes.items())},
                  "available_prefix_plan_sha256": score.prefix_digest.hexdigest(), "evaluation_seed": eval_seed,
                  "training_manifest_sha256": train_hash, "validation_manifest_sha256": sampler.manifest_hash,
                  "checkpoint": str(ckpt.resolve()), "checkpoint_manifest_sha256": _file_hash(ckpt / "manifest.json"),
                  "checkpoint_state_sha256": _file_hash(ckpt / "state.pt"), "checkpoint_progress": ckpt_progress,
                  "training_descriptor": descriptor, "operator_audit": model.operator_audit(),
                  "model_sha256": before_model,
                  "frozen_state": {"model_before": before_model, "model_after": after_model,
                                   "buffers_before": before_buffers, "buffers_after": after_buffers, "unchanged": True},
                  "sampler": {"initial": initial, "final": sampler.state_dict(), "rows_scanned": sampler.epoch_row_count,
                              "forwarded_batches": score.forward_batches},
                  "probe": {"context_override": context, "batch_size": 1, "device": str(dev),
                            "dtype": str(next(model.parameters()).dtype), "autocast": False,
                            **_source_provenance(ckpt_code), "torch_version": str(torch.__version__),
                            "deterministic_algorithms": torch.are_deterministic_algorithms_enabled()},
                  "exposure": {"split": "val", "unique_prediction_tokens": tokens,
                               "forward_input_tokens": score.forward_tokens, "final_test_exposed": False}}
        status = "complete"
    finally:
        ledger.finish(run_id, time.monotonic() - started, status)
    result["billing"] = json.loads(ledger.path.read_text())["runs"][run_id]
    (out_dir / "evaluation.json").write_text(json.dumps(result, indent=2, allow_nan=False) + "\n")
    return result


# ====================================================================================== paired comparison
def _require(condition, message):
    if not condition:
        raise ValueError(message)


def _check_frozen_proof(report):
    frozen = report.get("frozen_state", {})
    model_before = frozen.get("model_before")
    _require(frozen.get("unchanged") is True and model_before and model_before == frozen.get("model_after")
             and model_before == report.get("model_sha256") and frozen.get("buffers_before")
             and frozen.get("buffers_before") == frozen.get("buffers_after"),
             "evaluation lacks consistent frozen-state proof")


def _planned_counts(report) -> dict:
    """document id -> planned target count, after checking the plan's identity and shape."""
    plan = report.get("target_plan")
    _require(isinstance(plan, dict) and plan.get("split") == "val", "invalid validation target plan")
    _require(canonical_sha256(plan) == report.get("target_plan_sha256"), "target-plan SHA256 mismatch")
    _require(plan.get("validation_manifest_sha256")
             and plan["validation_manifest_sha256"] == report.get("validation_manifest_sha256"),
             "validation manifest identity mismatch")
    context, prefix_hash = report.get("context"), report.get("available_prefix_plan_sha256")
    _require(type(context) is int and context > 0 and isinstance(prefix_hash, str) and len(prefix_hash) == 64,
             "invalid context or prefix provenance")
    planned = {}
    for r in plan.get("ranges") or []:
        doc, start, end, count = (r.get(k) for k in ("document_id", "target_start", "target_end", "count"))
        _require(isinstance(doc, str) and doc not in planned and all(type(x) is int for x in (start, end, count))
                 and start >= 1 and end > start and count == end - start, "invalid or duplicate target range/count")
        planned[doc] = count
    _require(planned, "empty target plan")
    return planned


def _check_separation_audit(report, planned):
    audit = report.get("data_overlap_audit", {})
    _require(report.get("evaluation_protocol_version") == 2 and audit.get("has_overlap") is False
             and audit.get("training_manifest_hash") == report.get("training_manifest_sha256")
             and audit.get("validation_manifest_hash") == report.get("validation_manifest_sha256"),
             "evaluation lacks certified exact-document separation audit")
    ids = hashlib.sha256(json.dumps(sorted(planned), separators=(",", ":"), ensure_ascii=True).encode()).hexdigest()
    _require(audit.get("selected_validation_documents") == len(planned)
             and audit.get("selected_validation_ids_sha256") == ids, "document separation audit differs from target plan")


def _finite_loss(value) -> bool:
    return not isinstance(value, bool) and isinstance(value, (int, float)) and math.isfinite(value) and value >= 0


def _per_document(report, planned) -> dict:
    """document id -> (targets, loss sum), checked against the plan and the report's aggregates."""
    rows = {}
    for r in report.get("per_document") or []:
        doc, n, loss = r.get("document_id"), r.get("tokens"), r.get("loss_sum")
        _require(isinstance(doc, str) and doc not in rows and type(n) is int and n > 0 and _finite_loss(loss)
                 and planned.get(doc) == n, "invalid per-document ID/count/loss")
        rows[doc] = (n, float(loss))
    _require(set(rows) == set(planned), "per-document IDs differ from target plan")
    targets = sum(n for n, _ in rows.values())
    loss = sum(s for _, s in rows.values())
    close = lambda a, b: math.isclose(a, b, rel_tol=1e-12, abs_tol=1e-10)  # noqa: E731
    _require(report.get("prediction_tokens") == targets and close(report.get("loss_sum", -1), loss)
             and close(report.get("ce", -1), loss / targets), "aggregate losses/counts disagree with per-document state")
    return rows


def _validated_report(value):
    """A held-out evaluation report (or its path), checked for internal consistency; returns
    (report, per-document rows)."""
    report = json.loads(Path(value).read_text()) if isinstance(value, (str, Path)) else value
    _require(isinstance(report, dict) and report.get("kind") == "held_out_validation" and report.get("split") == "val",
             "comparison requires held_out_validation reports")
    _check_frozen_proof(report)
    planned = _planned_counts(report)
    _check_separation_audit(report, planned)
    return report, _per_document(report, planned)


_REPORT_IDENTITY = ("checkpoint", "checkpoint_manifest_sha256", "checkpoint_state_sha256", "checkpoint_progress",
                    "training_descriptor", "model_sha256", "operator_audit", "probe", "context", "evaluation_seed",
                    "available_prefix_plan_sha256", "available_prefix_length_histogram", "ce")


def compare_evaluations(left, right, out_dir, *, bootstrap_samples=1000, seed=0) -> dict:
    """Paired document bootstrap of CE_right - CE_left on identical target plans."""
    if type(bootstrap_samples) is not int or not 0 <= bootstrap_samples <= 100_000:
        raise ValueError("bootstrap_samples must be in [0, 100000]")
    if type(seed) is not int or seed < 0:
        raise ValueError("seed must be a nonnegative integer")
    left, left_docs = _validated_report(left)
    right, right_docs = _validated_report(right)
    if (left["target_plan"] != right["target_plan"]
            or left["validation_manifest_sha256"] != right["validation_manifest_sha256"]):
        raise ValueError("evaluations have different target plans or validation manifests")
    if set(left_docs) != set(right_docs) or any(left_docs[k][0] != right_docs[k][0] for k in left_docs):
        raise ValueError("evaluations have different per-document targets/counts")
    same_prefixes = left["available_prefix_plan_sha256"] == right["available_prefix_plan_sha256"]
    if left["context"] == right["context"] and not same_prefixes:
        raise ValueError("same-context evaluations have different available prefix plans")
    names = sorted(left_docs)
    counts = [left_docs[k][0] for k in names]
    deltas = [right_docs[k][1] - left_docs[k][1] for k in names]
    tokens = int(np.sum(counts, dtype=np.int64))
    ci = ratio_bootstrap(deltas, counts, samples=bootstrap_samples, seed=seed)
    result = {"kind": "matched_validation_comparison", "left": {k: left.get(k) for k in _REPORT_IDENTITY},
              "right": {k: right.get(k) for k in _REPORT_IDENTITY},
              "validation_manifest_sha256": left["validation_manifest_sha256"],
              "target_plan_sha256": left["target_plan_sha256"], "prediction_tokens": tokens, "documents": len(names),
              "contexts_match": left["context"] == right["context"], "available_prefix_plans_match": same_prefixes,
              "training_comparison": _training_comparison(left, right), "automatic_ranking_eligible": False,
              "prefix_comparison": ("identical available prefixes" if same_prefixes
                                    else "different available prefixes across contexts"),
              "delta_ce_right_minus_left": float(np.sum(deltas, dtype=np.float64) / tokens),
              "uncertainty": {"method": "paired document bootstrap of token-weighted CE difference",
                              "unit": "nominal document uncertainty; not training seeds or HPO correction",
                              "bootstrap_samples": bootstrap_samples, "seed": seed, "delta_ce_95_ci": ci},
              "interpretation": "matched-target predictive loss comparison; no automatic fair ranking"}
    if out_dir is None:
        return result
    out_dir = Path(out_dir)
    out_dir.mkdir(parents=True, exist_ok=False)
    (out_dir / "comparison.json").write_text(json.dumps(result, indent=2, allow_nan=False) + "\n")
    return result


def _gpt2():
    import tiktoken
    tok = tiktoken.get_encoding("gpt2")
    ranks = sorted((k.hex(), v) for k, v in tok._mergeable_ranks.items())
    fp = hashlib.sha256(json.dumps({"ranks": ranks, "regex_pattern": tok._pat_str,
                                    "special_tokens": tok._special_tokens}, sort_keys=True).encode()).hexdigest()
    return tok, fp


def evaluate_mechanisms(cfg, checkpoint, task_manifest, out_dir, *, max_examples=32, max_seconds=300, device="cpu",
                        components=("0:attn", "0:mlp"), run_budget_usd=None, max_prompt_tokens=None, tokenizer=None):
    """Answer-only exact-label probes with branch removal and final-position activation transfer.

    ``tokenizer`` defaults to GPT-2 (tiktoken) and must match the training data's fingerprint; an
    injected tokenizer (tests) must match an injected test-only training tokenizer by name."""
    from .analysis import reference_path
    from .checkpoint import load_checkpoint
    from .data import manifest_hash
    from .tasks import audit_mechanism_training, load_mechanism_tasks
    if isinstance(cfg, (str, Path)):
        cfg = Config.from_yaml(str(cfg))
    project = cfg.raw.get("project", {})
    components = tuple(components)
    cap = cfg.raw.get("data", {}).get("context", 512) if max_prompt_tokens is None else max_prompt_tokens
    if project.get("dry_run", True):
        return {"dry_run": True, "command": "evaluate_mechanisms", "checkpoint": str(checkpoint),
                "task_manifest": str(task_manifest), "max_examples": max_examples, "max_prompt_tokens": cap,
                "components": list(components)}
    if type(max_examples) is not int or max_examples <= 0 or type(cap) is not int or cap <= 0 \
            or not math.isfinite(max_seconds) or max_seconds <= 0:
        raise ValueError("positive bounded mechanism evaluation limits required")
    parsed = []
    for comp in components:
        try:
            layer, branch = comp.split(":")
            layer = int(layer)
        except (AttributeError, ValueError) as e:
            raise ValueError("component must be layer:attn or layer:mlp") from e
        if branch not in ("attn", "mlp") or not 0 <= layer < cfg.model.layers or comp in [c[0] for c in parsed]:
            raise ValueError("invalid or duplicate branch-removal component")
        parsed.append((comp, layer, branch))
    dev = torch.device(device)
    rate = project.get("gpu_hourly_rate_usd")
    if rate is None or (dev.type == "cuda" and rate <= 0):
        raise ValueError("declare actual gpu_hourly_rate_usd (explicit 0 allowed for CPU)")
    out_dir = Path(out_dir)
    if out_dir.exists():
        raise FileExistsError(f"mechanism evaluation directory already exists: {out_dir}")
    ledger = _ledger(project)
    run_id = str(out_dir.resolve())
    ledger.begin(run_id, rate, max_seconds, run_budget_usd, parent_checkpoint=checkpoint,
                 cost_margin_fraction=project.get("cost_margin_fraction", .1), stage=project.get("stage", "A"))
    started, status = time.monotonic(), "failed"

    def deadline():
        if time.monotonic() - started >= max_seconds:
            raise TimeoutError("mechanism evaluation runtime cap exhausted")

    try:
        out_dir.mkdir(parents=True, exist_ok=False)
        metadata, all_rows = load_mechanism_tasks(task_manifest, split="val")
        rows = all_rows[:max_examples]
        if not rows:
            raise ValueError("mechanism validation split is empty")
        task_hash = manifest_hash(task_manifest)
        train_manifest = cfg.raw["data"]["manifest"]
        training_hash = manifest_hash(train_manifest)
        train_tok = json.loads(Path(train_manifest, "manifest.json").read_text() if Path(train_manifest).is_dir()
                               else Path(train_manifest).read_text())["tokenizer"]
        if tokenizer is None:
            tokenizer, fp = _gpt2()
            if train_tok.get("fingerprint_sha256") != fp:
                raise ValueError("mechanism prompts require the checkpoint training GPT2 tokenizer fingerprint")
        elif not (train_tok.get("test_only") and train_tok.get("name") == getattr(tokenizer, "name", None)):
            raise ValueError("an injected tokenizer must match the test-only training tokenizer")
        exposure = audit_mechanism_training(task_manifest, train_manifest)
        encode = tokenizer.encode_ordinary if hasattr(tokenizer, "encode_ordinary") else tokenizer.encode
        cand = {}
        for task, digits in (("boolean_hierarchy", range(2)), ("associative_retrieval", range(4))):
            ids = [encode(f" {d}") for d in digits]
            if any(len(t) != 1 for t in ids):
                raise ValueError("mechanism candidate answers must be exactly one token")
            cand[task] = [t[0] for t in ids]
        encoded = []
        for r in rows:
            prompt, answer = encode(r["prompt"]), encode(r["answer"])
            if len(answer) != 1 or answer[0] not in cand[r["task"]]:
                raise ValueError("mechanism answer must be exactly one task-candidate token")
            if not prompt or len(prompt) > cap:
                raise ValueError("mechanism prompt exceeds explicit context cap; no truncation permitted")
            if max(prompt + answer) >= cfg.model.vocab_size:
                raise ValueError("mechanism tokens exceed checkpoint vocabulary")
            encoded.append((r, prompt, answer[0]))
        model = TensorLM(cfg.model)
        payload = load_checkpoint(checkpoint, model, expected_manifest_hash=training_hash,
                                  config_validator=evaluation_validator(cfg), restore_rng=False, map_location="cpu")
        progress, code = payload["progress"], payload["code"]
        descriptor = _training_descriptor(payload)
        del payload
        model.to(dev).eval()
        for norm in lagged_modules(model):
            _check_lagged_divisor(norm)
        before_p, before_b = _tensor_hash(model.named_parameters()), _tensor_hash(model.named_buffers())
        fwd_tokens = [0]

        def score(prompt, answer, task):
            deadline()
            idx = torch.tensor([prompt], dtype=torch.long, device=dev)
            logits = model(idx, doc_ids=torch.zeros_like(idx))[0, -1].float()
            if not bool(torch.isfinite(logits).all()):
                raise FloatingPointError("nonfinite mechanism logits")
            ce = float(F.cross_entropy(logits[None], torch.tensor([answer], device=dev)))
            pred = int(logits.argmax())
            constrained = cand[task][int(logits[cand[task]].argmax())]
            fwd_tokens[0] += len(prompt)
            return {"answer_ce": ce, "full_vocab_prediction_token": pred, "full_vocab_correct": pred == answer,
                    "candidate_prediction_token": constrained, "candidate_correct": constrained == answer}

        def delta(measured, base):
            measured["delta_answer_ce"] = measured["answer_ce"] - base["answer_ce"]
            measured["delta_full_vocab_correct"] = int(measured["full_vocab_correct"]) - int(base["full_vocab_correct"])
            measured["delta_candidate_correct"] = int(measured["candidate_correct"]) - int(base["candidate_correct"])
            return measured

        examples, cached, reuse_count = [], {}, 0
        with reference_path(model), torch.inference_mode():
            for r, prompt, answer in encoded:
                caps, handles = {}, []
                for name, layer, branch in parsed:
                    def hook(module, inputs, output, name=name):
                        caps[name] = output[0, -1].detach().cpu().clone()
                    handles.append(getattr(model.blocks[layer], branch).register_forward_hook(hook))
                try:
                    base = score(prompt, answer, r["task"])
                finally:
                    for h in handles:
                        h.remove()
                cached[r["id"]] = caps
                contrasts = {}
                for name, layer, branch in parsed:
                    model.blocks[layer].ablate = frozenset({branch})
                    try:
                        contrasts[name] = delta(score(prompt, answer, r["task"]), base)
                    finally:
                        model.blocks[layer].ablate = frozenset()
                examples.append({"id": r["id"], "task": r["task"], "composition_id": r["composition_id"],
                                 "prompt": r["prompt"], "answer": r["answer"], "answer_token": answer,
                                 "prompt_tokens": len(prompt), "baseline": base, "branch_removal": contrasts})
            for target, (r, prompt, answer) in zip(examples, encoded):
                target["branch_reuse"] = {}
                for name, layer, branch in parsed:
                    transfers = {}
                    for donor_class in ("same_answer", "different_answer"):
                        eligible = [c for c in rows if c["task"] == r["task"] and c["composition_id"] != r["composition_id"]
                                    and ((c["answer"] == r["answer"]) == (donor_class == "same_answer"))]
                        if not eligible:
                            transfers[donor_class] = {"status": "skipped", "reason": "no eligible donor"}
                            continue
                        donor = min(eligible, key=lambda c: c["id"])
                        vec = cached[donor["id"]][name]

                        def patch(module, inputs, output, vec=vec):
                            out = output.clone()
                            out[0, -1] = vec.to(device=output.device, dtype=output.dtype)
                            return out
                        h = getattr(model.blocks[layer], branch).register_forward_hook(patch)
                        try:
                            m = delta(score(prompt, answer, r["task"]), target["baseline"])
                        finally:
                            h.remove()
                        reuse_count += 1
                        m.update(status="patched", donor_id=donor["id"], donor_composition_id=donor["composition_id"],
                                 donor_answer=donor["answer"])
                        transfers[donor_class] = m
                    target["branch_reuse"][name] = transfers
        if (before_p, before_b) != (_tensor_hash(model.named_parameters()), _tensor_hash(model.named_buffers())):
            raise RuntimeError("mechanism evaluation mutated checkpoint parameters/buffers")

        def summarize(sel):
            n = len(sel)
            met = lambda vals: {"answer_ce": sum(v["answer_ce"] for v in vals) / n,  # noqa: E731
                                "full_vocab_accuracy": sum(v["full_vocab_correct"] for v in vals) / n,
                                "candidate_accuracy": sum(v["candidate_correct"] for v in vals) / n}
            out = {"examples": n, "baseline": met([s["baseline"] for s in sel]), "branch_removal": {}, "branch_reuse": {}}
            for name in components:
                vals = [s["branch_removal"][name] for s in sel]
                out["branch_removal"][name] = {**met(vals),
                                               "paired_mean_delta_answer_ce": sum(v["delta_answer_ce"] for v in vals) / n}
                out["branch_reuse"][name] = {}
                for dc in ("same_answer", "different_answer"):
                    patched = [s["branch_reuse"][name][dc] for s in sel if s["branch_reuse"][name][dc]["status"] == "patched"]
                    summ = {"patched_examples": len(patched), "skipped_examples": n - len(patched)}
                    if patched:
                        summ["paired_mean_delta_answer_ce"] = sum(v["delta_answer_ce"] for v in patched) / len(patched)
                        summ["candidate_accuracy"] = sum(v["candidate_correct"] for v in patched) / len(patched)
                    out["branch_reuse"][name][dc] = summ
            return out

        ckpt = Path(checkpoint)
        result = {"kind": "known_mechanism_evaluation", "split": "val", "examples": examples,
                  "summary": summarize(examples),
                  "per_task": {t: summarize([e for e in examples if e["task"] == t]) for t in sorted({e["task"] for e in examples})},
                  "probe_ids": [e["id"] for e in examples], "task_manifest_sha256": task_hash, "task_metadata": metadata,
                  "training_manifest_sha256": training_hash, "checkpoint": str(ckpt.resolve()),
                  "checkpoint_manifest_sha256": _file_hash(ckpt / "manifest.json"),
                  "checkpoint_state_sha256": _file_hash(ckpt / "state.pt"), "checkpoint_progress": progress,
                  "training_descriptor": descriptor, "checkpoint_code": code, "operator_audit": model.operator_audit(),
                  "probe": {"device": str(dev), "max_examples": max_examples, "max_prompt_tokens": cap,
                            "components": list(components), "autocast": False, "candidate_token_ids": cand},
                  "frozen_state": {"unchanged": True, "parameters": before_p, "buffers": before_b},
                  "exposure": {"answer_prediction_tokens": len(examples) * (1 + len(components)),
                               "reuse_answer_prediction_tokens": reuse_count, "forward_input_tokens": fwd_tokens[0],
                               "final_test_exposed": False},
                  "generator_composition_holdout_verified": True,
                  "benchmark_training_exposure_verified": exposure["verified"], "training_exposure_audit": exposure,
                  "interpretation": "exact-label task evidence, not an LM-quality proxy or unique causal mediation claim"}
        status = "complete"
    finally:
        ledger.finish(run_id, time.monotonic() - started, status)
    result["billing"] = json.loads(ledger.path.read_text())["runs"][run_id]
    tmp = out_dir / ".mechanism_evaluation.json.tmp"
    tmp.write_text(json.dumps(result, indent=2, allow_nan=False) + "\n")
    os.replace(tmp, out_dir / "mechanism_evaluation.json")
    return result
