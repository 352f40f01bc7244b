"""Optimizer exposure: what the learning-rate and decoupled-decay schedule has applied so far.

For every optimizer group the record keeps the number of updates observed, the sum of the group's
learning rates, the sum of lr * weight_decay, and the shrinkage product prod(1 - lr*wd) that
decoupled decay multiplies a weight by, kept as (sign, log|product|, count of exact zeros) so it
neither under- nor overflows.  The numbers describe a parameter that took part in every update (AdamW
and Muon decay only parameters that received a gradient) and, for Muon, the raw group LR its decay
uses (its orthogonalised update has a separate shape-adjusted LR).

The record lives in ``progress["optimizer_exposure"]`` and travels in checkpoints, so its schema and
the group identity digest (sha256 of ``json.dumps(identity, sort_keys=True)``) are the reference's
(tnlm/optimizer_exposure.py:31-104): either framework continues the other's totals on resume.
Observation never changes the optimizer.
"""
from __future__ import annotations

import copy
import hashlib
import json
import math
from typing import NamedTuple

import torch

from .optim import FusedAdamW, Muon, MuonAdamW

SCOPE = ("scheduled group exposure; mathematical shrinkage product before floating-point rounding, for a "
         "parameter participating in every observed update")
MUON_DECAY = "raw group lr; Newton-Schulz update separately shape-adjusted"


class _Group(NamedTuple):
    identity: dict
    digest: str
    lr: float
    lr_wd: float


def _nonnegative(value, what: str) -> float:
    if isinstance(value, torch.Tensor):
        if value.numel() != 1:
            raise ValueError(f"{what} must be a scalar")
        value = value.item()
    value = float(value)
    if not (math.isfinite(value) and value >= 0):
        raise ValueError(f"{what} must be finite and nonnegative")
    return value


def _is_adamw(optimizer) -> bool:
    """torch AdamW or its fused-kernel subclass (same hyper-parameters and update rule)."""
    return type(optimizer) in (torch.optim.AdamW, FusedAdamW)


def _parts(optimizer) -> list[tuple[str, torch.optim.Optimizer]]:
    if _is_adamw(optimizer):
        return [("adamw", optimizer)]
    if (type(optimizer) is MuonAdamW and isinstance(optimizer.muon, (Muon, torch.optim.Muon))
            and _is_adamw(optimizer.adamw)):
        return [("muon", optimizer.muon), ("adamw", optimizer.adamw)]
    raise ValueError("optimizer exposure is defined for AdamW and MuonAdamW only")


def _groups(optimizer) -> list[_Group]:
    out = []
    for kind, part in _parts(optimizer):
        for g in part.param_groups:
            identity = {"index": len(out), "optimizer_kind": kind, "kind": g.get("kind"),
                        "parameters": [{"shape": list(p.shape), "dtype": str(p.dtype)} for p in g["params"]],
                        "parameter_names": copy.deepcopy(g.get("param_names"))}
            digest = hashlib.sha256(json.dumps(identity, sort_keys=True, allow_nan=False).encode()).hexdigest()
            lr = _nonnegative(g["lr"], "lr")
            lr_wd = lr * _nonnegative(g.get("weight_decay", 0.0), "weight_decay")
            if not math.isfinite(lr_wd):
                raise ValueError("lr * weight_decay is not finite")
            out.append(_Group(identity, digest, lr, lr_wd))
    return out


def _empty(groups: list[_Group], steps: int, tokens: int) -> dict:
    return {"version": 1, "complete_history": steps == 0 and tokens == 0, "known_start_steps": steps,
            "known_start_tokens": tokens, "observed_steps": 0, "scope": SCOPE, "muon_decay_semantics": MUON_DECAY,
            "groups": [{"identity": g.identity, "identity_sha256": g.digest, "observed_steps": 0, "sum_lr": 0.0,
                        "sum_lr_weight_decay": 0.0, "sum_log_abs_nonzero_factors": 0.0, "zero_factors": 0,
                        "negative_factors": 0, "shrinkage_sign": 1, "shrinkage_log_abs": 0.0} for g in groups]}


def _add_update(row: dict, g: _Group) -> None:
    row["observed_steps"] += 1
    row["sum_lr"] += g.lr
    row["sum_lr_weight_decay"] += g.lr_wd
    factor = 1.0 - g.lr_wd
    if factor == 0.0:
        row["zero_factors"] += 1
    else:
        # log1p keeps precision for the usual tiny lr*wd; a negative factor flips the sign
        row["sum_log_abs_nonzero_factors"] += math.log1p(-g.lr_wd) if factor > 0 else math.log(-factor)
        if factor < 0:
            row["negative_factors"] += 1
    if row["zero_factors"]:
        row["shrinkage_sign"], row["shrinkage_log_abs"] = 0, None
    else:
        row["shrinkage_sign"] = -1 if row["negative_factors"] % 2 else 1
        row["shrinkage_log_abs"] = row["sum_log_abs_nonzero_factors"]


def update_optimizer_exposure(progress: dict, optimizer) -> dict:
    """Count one completed update.  Call after ``optimizer.step()`` and before the progress counters
    advance.  Everything is checked on a copy; ``progress`` changes only if all of it holds."""
    steps, tokens = progress.get("steps", 0), progress.get("tokens", 0)
    if any(isinstance(v, bool) or not isinstance(v, int) or v < 0 for v in (steps, tokens)):
        raise ValueError("progress steps and tokens must be nonnegative integers")
    groups = _groups(optimizer)
    prior = progress.get("optimizer_exposure")
    if prior is None:
        record = _empty(groups, steps, tokens)
    else:
        record = copy.deepcopy(prior)
        if record.get("version") != 1 or len(record["groups"]) != len(groups):
            raise ValueError("the recorded optimizer exposure has another schema or group count")
        if record["known_start_steps"] + record["observed_steps"] != steps:
            raise ValueError("the recorded optimizer exposure does not end at the current step")
    for row, g in zip(record["groups"], groups):
        if row["identity_sha256"] != g.digest or row["identity"] != g.identity:
            raise ValueError(f"optimizer group {g.identity['index']} is not the group the exposure recorded")
        _add_update(row, g)
    record["observed_steps"] += 1
    try:  # overflowed or corrupted totals must fail before progress is touched
        json.dumps(record, allow_nan=False)
    except (ValueError, TypeError) as exc:
        raise ValueError("the optimizer exposure is no longer finite JSON") from exc
    progress["optimizer_exposure"] = record
    return record
