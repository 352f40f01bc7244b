"""Per-group optimizer exposure bookkeeping: sum of learning rates, sum of lr * weight_decay and
the log of the decoupled-decay shrinkage product (reference tnlm/optimizer_exposure.py:31-104).
Observes group settings only; never changes the optimizer."""
from __future__ import annotations

import copy
import hashlib
import json
import math

import torch

from .optim import Muon, MuonAdamW


def _scalar(value, name) -> float:
    if isinstance(value, torch.Tensor):
        if value.numel() != 1:
            raise ValueError(f"{name} must be scalar")
        value = value.item()
    value = float(value)
    if not math.isfinite(value) or value < 0:
        raise ValueError(f"{name} must be finite and nonnegative")
    return value


def _children(optimizer):
    if type(optimizer) is torch.optim.AdamW:
        return [("adamw", optimizer)]
    if type(optimizer) is MuonAdamW and isinstance(optimizer.muon, (Muon, torch.optim.Muon)) \
            and type(optimizer.adamw) is torch.optim.AdamW:
        return [("muon", optimizer.muon), ("adamw", optimizer.adamw)]
    raise ValueError("exposure supports exactly AdamW and MuonAdamW")


def update_optimizer_exposure(progress: dict, optimizer) -> dict:
    """Record one completed update (call after optimizer.step, before advancing progress)."""
    steps, tokens = progress.get("steps", 0), progress.get("tokens", 0)
    if any(isinstance(v, bool) or not isinstance(v, int) or v < 0 for v in (steps, tokens)):
        raise ValueError("progress steps/tokens must be nonnegative integers")
    groups = []
    for kind, child in _children(optimizer):
        for group in child.param_groups:
            identity = {"index": len(groups), "optimizer_kind": kind, "kind": group.get("kind"),
                        "parameters": [{"shape": list(p.shape), "dtype": str(p.dtype)} for p in group["params"]],
                        "parameter_names": copy.deepcopy(group.get("param_names"))}
            digest = hashlib.sha256(json.dumps(identity, sort_keys=True, allow_nan=False).encode()).hexdigest()
            lr = _scalar(group["lr"], "lr")
            prod = lr * _scalar(group.get("weight_decay", 0.0), "weight_decay")
            if not math.isfinite(prod):
                raise ValueError("lr*weight_decay must be finite")
            groups.append((identity, digest, lr, prod))
    previous = progress.get("optimizer_exposure")
    if previous is None:
        exposure = {"version": 1, "complete_history": steps == 0 and tokens == 0, "known_start_steps": steps,
                    "known_start_tokens": tokens, "observed_steps": 0,
                    "scope": "scheduled group exposure; mathematical shrinkage product before floating-point "
                             "rounding, for a parameter participating in every observed update",
                    "muon_decay_semantics": "raw group lr; Newton-Schulz update separately shape-adjusted",
                    "groups": [{"identity": i, "identity_sha256": d, "observed_steps": 0, "sum_lr": 0.0,
                                "sum_lr_weight_decay": 0.0, "sum_log_abs_nonzero_factors": 0.0, "zero_factors": 0,
                                "negative_factors": 0, "shrinkage_sign": 1, "shrinkage_log_abs": 0.0}
                               for i, d, _, _ in groups]}
    else:
        exposure = copy.deepcopy(previous)
        if exposure.get("version") != 1 or len(exposure["groups"]) != len(groups):
            raise ValueError("optimizer exposure schema/group mismatch")
        if exposure["known_start_steps"] + exposure["observed_steps"] != steps:
            raise ValueError("optimizer exposure step history mismatch")
    for rec, (identity, digest, lr, prod) in zip(exposure["groups"], groups):
        if rec["identity_sha256"] != digest or rec["identity"] != identity:
            raise ValueError("optimizer exposure group identity mismatch")
        rec["sum_lr"] += lr
        rec["sum_lr_weight_decay"] += prod
        rec["observed_steps"] += 1
        factor = 1.0 - prod
        if factor == 0:
            rec["zero_factors"] += 1
        else:
            rec["sum_log_abs_nonzero_factors"] += math.log1p(-prod) if factor > 0 else math.log(-factor)
            rec["negative_factors"] += int(factor < 0)
        rec["shrinkage_sign"] = 0 if rec["zero_factors"] else (-1 if rec["negative_factors"] % 2 else 1)
        rec["shrinkage_log_abs"] = None if rec["zero_factors"] else rec["sum_log_abs_nonzero_factors"]
    exposure["observed_steps"] += 1
    try:
        json.dumps(exposure, allow_nan=False)
    except (ValueError, TypeError) as exc:
        raise ValueError("optimizer exposure must remain finite JSON") from exc
    progress["optimizer_exposure"] = exposure
    return exposure
