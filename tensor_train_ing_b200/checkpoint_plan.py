"""Checkpoint retention policy, milestone schedule and a meta-device storage forecast
(reference tnlm/checkpoint_plan.py:24-213).  Nothing is allocated, written or deleted."""
from __future__ import annotations

import bisect
import heapq
import math

import torch

from .optim import hidden_matrix

_METADATA_ALLOWANCE = 1 << 20
_SERIALIZATION_OVERHEAD = 1 << 20
_EARLY = (1_000_000, 2_000_000, 4_000_000, 8_000_000, 16_000_000, 32_000_000)


def _integer(value, name, minimum=0):
    if isinstance(value, bool) or not isinstance(value, int) or value < minimum:
        raise ValueError(f"{name} must be an integer >= {minimum}")
    return value


def checkpoint_retention_policy(cfg) -> dict:
    project = cfg.raw.get("project", {})
    keep = _integer(project.get("keep_recovery_checkpoints", 2), "project.keep_recovery_checkpoints")
    initial = project.get("save_initial_checkpoint", True)
    if not isinstance(initial, bool):
        raise ValueError("project.save_initial_checkpoint must be bool")
    return {"keep_recovery_checkpoints": keep, "save_initial_checkpoint": initial}


def milestone_policy(cfg) -> dict:
    project = cfg.raw.get("project", {})
    if "milestone_tokens" not in project:
        return {"mode": "default", "tokens": None}
    values = project["milestone_tokens"]
    if not isinstance(values, list):
        raise ValueError("project.milestone_tokens must be a list of positive integers")
    for v in values:
        _integer(v, "project.milestone_tokens entry", 1)
    return {"mode": "explicit", "tokens": sorted(set(values))}


def pending_milestone_tokens(cfg, *, start_tokens, token_limit, reachable_tokens=None, include_branch=False):
    """Lazy, sorted, unique milestone thresholds in (start, min(limit, reachable)]; the default is
    1M..32M doubling then every 100M; ``include_branch`` adds the 90% branch point."""
    start = _integer(start_tokens, "start_tokens")
    limit = _integer(token_limit, "token_limit")
    end = limit if reachable_tokens is None else min(limit, _integer(reachable_tokens, "reachable_tokens"))
    if not isinstance(include_branch, bool):
        raise ValueError("include_branch must be bool")
    policy = milestone_policy(cfg)
    if policy["mode"] == "explicit":
        vals = policy["tokens"]
        sources = [iter(vals[bisect.bisect_right(vals, start):bisect.bisect_right(vals, end)])]
    else:
        sources = [(v for v in _EARLY if start < v <= end),
                   range((start // 100_000_000 + 1) * 100_000_000, end + 1, 100_000_000)]
    branch = (9 * limit) // 10
    if include_branch and cfg.train.schedule != "cosine" and start < branch <= end:
        sources.append((branch,))

    def unique():
        prev = None
        for v in heapq.merge(*sources):
            if v != prev:
                yield v
                prev = v
    return unique()


def checkpoint_storage_plan(cfg, *, start_tokens=0, token_limit=None, max_steps=None, distributed_world_size=1,
                            distributed=False, export_weights=False, cooldown=False) -> dict:
    """Advisory bytes for all checkpoints the run will retain, from a meta-device model."""
    from .models.model import TensorLM
    start = _integer(start_tokens, "start_tokens")
    limit = _integer(cfg.train.rung_total_tokens if token_limit is None else token_limit, "token_limit")
    world = _integer(distributed_world_size, "distributed_world_size", 1)
    if not distributed and world != 1:
        raise ValueError("distributed_world_size must be 1 for a serial plan")
    for name, v in (("distributed", distributed), ("export_weights", export_weights), ("cooldown", cooldown)):
        if not isinstance(v, bool):
            raise ValueError(f"{name} must be bool")
    batch = _integer(cfg.train.global_prediction_tokens_per_update, "global_prediction_tokens_per_update", 1)
    retention = checkpoint_retention_policy(cfg)
    keep = retention["keep_recovery_checkpoints"]
    updates = (max(0, limit - start) + batch - 1) // batch
    if max_steps is not None:
        updates = min(updates, _integer(max_steps, "max_steps"))
    reachable = min(limit, start + updates * batch) if start < limit else start
    policy = milestone_policy(cfg)
    end = min(limit, reachable)
    if policy["mode"] == "default":
        milestones = sum(start < v <= end for v in _EARLY) + max(0, end // 100_000_000 - start // 100_000_000)
    else:
        vals = policy["tokens"]
        milestones = max(0, bisect.bisect_right(vals, end) - bisect.bisect_right(vals, start))
    branch = (9 * limit) // 10
    branch_reachable = not cooldown and cfg.train.schedule != "cosine" and start < branch <= end
    branch_is_milestone = (branch in policy["tokens"] if policy["mode"] == "explicit"
                           else branch in _EARLY or (branch > 0 and branch % 100_000_000 == 0))
    separate_branch = int(branch_reachable and distributed)
    if branch_reachable and not distributed and not branch_is_milestone:
        milestones += 1
    rolling = min(updates, keep + 1) if keep else 0

    class _Meta(TensorLM):
        def reset_parameters(self):
            pass

    with torch.device("meta"):
        model = _Meta(cfg.model)
    if cfg.train.optimizer not in ("adamw", "muon"):
        raise ValueError("checkpoint plan supports adamw or muon")
    seen, param_bytes, opt_bytes, padding, step_scalars = set(), 0, 0, 0, 0
    for name, p in model.named_parameters():
        key = id(p)
        if key not in seen:
            seen.add(key)
            param_bytes += p.numel() * p.element_size()
        if not p.requires_grad:
            continue
        moments = 1 if cfg.train.optimizer == "muon" and hidden_matrix(name, p) else 2
        opt_bytes += moments * p.numel() * p.element_size()
        if moments == 2:
            step_scalars += 8 * world
        if distributed:
            row = (math.prod(p.shape[1:]) if p.ndim else p.numel()) * p.element_size()
            padding += (world - 1) * row * (1 + moments)
    portable = param_bytes
    buffers = sum(t.numel() * t.element_size() for n, t in model.state_dict().items()
                  if n not in dict(model.named_parameters())) * (world if distributed else 1)
    tensor_bytes = param_bytes + opt_bytes + step_scalars + padding + buffers

    def estimate(tensors, copies):
        base = tensors + _METADATA_ALLOWANCE * copies
        return base + (base + 9) // 10 + _SERIALIZATION_OVERHEAD * copies

    full = estimate(tensor_bytes, world if distributed else 1)
    export = estimate(portable + buffers // (world if distributed else 1), 1) if export_weights else 0
    counts = {"initial": int(retention["save_initial_checkpoint"]), "final": 1, "milestones": milestones,
              "separate_90_percent_branch": separate_branch, "rolling_recovery_including_staging": rolling}
    count = sum(counts.values())
    return {"kind": "checkpoint_storage_projection", "required_additional_bytes": full * count + export,
            "per_checkpoint_estimate_bytes": full, "export_weights_estimate_bytes": export, "checkpoint_count": count,
            "count_breakdown": counts, "milestone_policy": policy, "checkpoint_retention_policy": retention,
            "start_tokens": start, "token_limit": limit, "reachable_tokens": reachable, "reachable_updates": updates,
            "distributed": distributed, "world_size": world, "dtype": str(torch.get_default_dtype()),
            "tensor_bytes_breakdown": {"parameters": param_bytes, "optimizer_moments": opt_bytes,
                                       "optimizer_step_scalars": step_scalars, "persistent_buffers": buffers,
                                       "distributed_shard_padding_allowance": padding},
            "metadata_allowance_bytes_per_rank_checkpoint": _METADATA_ALLOWANCE,
            "scope": "advisory projection, not guaranteed upper bound; no reservation or deletion"}
