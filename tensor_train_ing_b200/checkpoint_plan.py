"""Checkpoint retention, the milestone schedule and a disk forecast for a planned run.

The forecast is computed from the model's shapes on the meta device: nothing is allocated,
initialised, drawn from an RNG, written, reserved or deleted.  Policies and numbers are the
reference planner's (tnlm/checkpoint_plan.py:24-213), field for field, because sweep journals and
run directories record these plans and the two frameworks' tools read each other's:

* retention: ``project.keep_recovery_checkpoints`` (default 2; 0 turns recovery saves off) and
  ``project.save_initial_checkpoint`` (default true); final, milestone and branch checkpoints stay;
* milestones: by default 1M, 2M, 4M, ... 32M tokens, then every 100M; an explicit
  ``project.milestone_tokens`` list replaces the whole default; the serial trainer also saves at the
  90 % branch point of a non-cosine schedule, the distributed trainer keeps it as its own checkpoint;
* one full-state checkpoint = parameters + optimizer moments (one per Muon matrix, two per AdamW
  tensor) + an 8-byte step per AdamW tensor per rank + persistent buffers, plus under sharding an
  allowance for uneven first-dimension splits, plus 1 MiB of metadata per rank file; then a 10 %
  serialisation margin and 1 MiB per rank file.
"""
from __future__ import annotations

import bisect
import heapq
import math
from dataclasses import dataclass
from typing import Iterator

import torch

from .optim import hidden_matrix

MIB = 1 << 20
METADATA_ALLOWANCE = MIB      # per rank checkpoint file
SERIALIZATION_OVERHEAD = MIB  # per rank checkpoint file, after the 10 % margin
STEP_SCALAR_BYTES = 8         # AdamW's step counter per tensor (at least; the default dtype if wider)


def _count(value, what: str, minimum: int = 0) -> int:
    if isinstance(value, bool) or not isinstance(value, int) or value < minimum:
        raise ValueError(f"{what} must be an integer >= {minimum}")
    return value


def _flag(value, what: str) -> bool:
    if not isinstance(value, bool):
        raise ValueError(f"{what} must be bool")
    return value


def checkpoint_retention_policy(cfg) -> dict:
    project = cfg.raw.get("project", {})
    return {"keep_recovery_checkpoints": _count(project.get("keep_recovery_checkpoints", 2),
                                                "project.keep_recovery_checkpoints"),
            "save_initial_checkpoint": _flag(project.get("save_initial_checkpoint", True),
                                             "project.save_initial_checkpoint")}


class MilestoneSchedule:
    """Token counts at which a milestone checkpoint is saved."""

    DOUBLING = (1_000_000, 2_000_000, 4_000_000, 8_000_000, 16_000_000, 32_000_000)
    STRIDE = 100_000_000

    def __init__(self, explicit: list[int] | None = None):
        self.explicit = explicit  # sorted unique values, or None for the default schedule

    @classmethod
    def from_config(cls, cfg) -> "MilestoneSchedule":
        project = cfg.raw.get("project", {})
        if "milestone_tokens" not in project:
            return cls()
        values = project["milestone_tokens"]
        if not isinstance(values, list):
            raise ValueError("project.milestone_tokens must be a list of positive integers")
        return cls(sorted({_count(v, "each project.milestone_tokens entry", 1) for v in values}))

    def policy(self) -> dict:
        return ({"mode": "default", "tokens": None} if self.explicit is None
                else {"mode": "explicit", "tokens": list(self.explicit)})

    def between(self, start: int, end: int) -> Iterator[int]:
        """Thresholds t with start < t <= end, ascending, produced lazily."""
        if self.explicit is not None:
            lo, hi = bisect.bisect_right(self.explicit, start), bisect.bisect_right(self.explicit, end)
            yield from self.explicit[lo:hi]
            return
        early = [t for t in self.DOUBLING if start < t <= end]
        strided = range((start // self.STRIDE + 1) * self.STRIDE, end + 1, self.STRIDE)
        yield from heapq.merge(early, strided)

    def count(self, start: int, end: int) -> int:
        if self.explicit is not None:
            return max(0, bisect.bisect_right(self.explicit, end) - bisect.bisect_right(self.explicit, start))
        early = sum(start < t <= end for t in self.DOUBLING)
        return early + max(0, end // self.STRIDE - start // self.STRIDE)

    def __contains__(self, tokens: int) -> bool:
        if self.explicit is not None:
            return tokens in self.explicit
        return tokens in self.DOUBLING or (tokens > 0 and tokens % self.STRIDE == 0)


def milestone_policy(cfg) -> dict:
    return MilestoneSchedule.from_config(cfg).policy()


def branch_point(limit: int) -> int:
    """The 90 % point of a token horizon, where sweeps branch their cooldowns."""
    return (9 * limit) // 10


def pending_milestone_tokens(cfg, *, start_tokens, token_limit, reachable_tokens=None, include_branch=False):
    """Unique thresholds in (start, min(limit, reachable)], ascending; with ``include_branch`` the 90 %
    branch point of a non-cosine schedule joins them.  Arguments are checked at the call, the values
    are produced lazily (the default schedule can span many 100M strides)."""
    start = _count(start_tokens, "start_tokens")
    limit = _count(token_limit, "token_limit")
    end = limit if reachable_tokens is None else min(limit, _count(reachable_tokens, "reachable_tokens"))
    _flag(include_branch, "include_branch")
    sources = [MilestoneSchedule.from_config(cfg).between(start, end)]
    bp = branch_point(limit)
    if include_branch and cfg.train.schedule != "cosine" and start < bp <= end:
        sources.append(iter((bp,)))

    def deduplicated():
        last = None
        for t in heapq.merge(*sources):
            if t != last:
                last = t
                yield t
    return deduplicated()


@dataclass
class _Inventory:
    """Tensor bytes of one full-state checkpoint of the model (all ranks together when sharded)."""
    parameters: int = 0            # unique storages; every FQN when sharded (DCP addresses by name)
    portable_parameters: int = 0   # unique storages (a torch.save export)
    moments: int = 0
    step_scalars: int = 0
    padding: int = 0               # uneven Shard(0) split allowance, model and moments
    buffers: int = 0               # persistent buffers, once per rank when sharded
    unique_buffers: int = 0

    def tensor_bytes(self) -> int:
        return self.parameters + self.moments + self.step_scalars + self.padding + self.buffers


def _inventory(cfg, world: int, sharded: bool) -> _Inventory:
    with torch.device("meta"):
        from .models.model import TensorLM
        model = TensorLM(cfg.model)
    inv = _Inventory()
    step_bytes = max(STEP_SCALAR_BYTES, torch.empty((), device="meta").element_size())
    storages = set()
    for name, p in model.named_parameters():
        key = p.untyped_storage()._cdata
        if key not in storages:
            storages.add(key)
            inv.portable_parameters += p.untyped_storage().nbytes()
        if not p.requires_grad:
            continue
        copies = 1 if cfg.train.optimizer == "muon" and hidden_matrix(name, p) else 2
        inv.moments += copies * p.numel() * p.element_size()
        if copies == 2:
            inv.step_scalars += step_bytes * world
        if sharded:
            # one first-dimension row per extra rank (whole tensor for a scalar), model and moments
            row = (math.prod(p.shape[1:]) if p.ndim else p.numel()) * p.element_size()
            inv.padding += (world - 1) * row * (1 + copies)
    inv.parameters = inv.portable_parameters
    if sharded:
        seen, inv.parameters = set(), 0
        for _, p in model.named_parameters(remove_duplicate=False):
            inv.parameters += p.numel() * p.element_size()
            if id(p) in seen:  # a tied parameter is saved (and padded) under each name
                inv.padding += (world - 1) * (math.prod(p.shape[1:]) if p.ndim else 1) * p.element_size()
            seen.add(id(p))
    param_keys = {p.untyped_storage()._cdata for p in model.parameters()}
    buffer_sizes = {}
    for t in model.state_dict().values():
        key = t.untyped_storage()._cdata
        if key not in param_keys:
            buffer_sizes[key] = t.untyped_storage().nbytes()
    inv.unique_buffers = sum(buffer_sizes.values())
    inv.buffers = inv.unique_buffers * (world if sharded else 1)
    return inv


def _on_disk(tensor_bytes: int, files: int) -> int:
    base = tensor_bytes + METADATA_ALLOWANCE * files
    return base + (base + 9) // 10 + SERIALIZATION_OVERHEAD * files


def checkpoint_storage_plan(cfg, *, start_tokens=0, token_limit=None, max_steps=None, distributed_world_size=1,
                            distributed=False, export_weights=False, cooldown=False) -> dict:
    """Advisory bytes of every checkpoint the run keeps at its peak (not a guaranteed bound:
    existing artifacts, concurrent runs and filesystem allocation are outside it)."""
    start = _count(start_tokens, "start_tokens")
    limit = _count(cfg.train.rung_total_tokens if token_limit is None else token_limit, "token_limit")
    world = _count(distributed_world_size, "distributed_world_size", 1)
    for value, what in ((distributed, "distributed"), (export_weights, "export_weights"), (cooldown, "cooldown")):
        _flag(value, what)
    if not distributed and world != 1:
        raise ValueError("a serial plan has distributed_world_size 1")
    batch = _count(cfg.train.global_prediction_tokens_per_update, "global_prediction_tokens_per_update", 1)
    if cfg.train.optimizer not in ("adamw", "muon"):
        raise ValueError("checkpoint plans cover the adamw and muon optimizers")
    retention = checkpoint_retention_policy(cfg)
    schedule = MilestoneSchedule.from_config(cfg)

    updates = -(-max(0, limit - start) // batch)
    if max_steps is not None:
        updates = min(updates, _count(max_steps, "max_steps"))
    reachable = min(limit, start + updates * batch) if start < limit else start
    end = min(limit, reachable)
    milestones = schedule.count(start, end)
    bp = branch_point(limit)
    branch_due = not cooldown and cfg.train.schedule != "cosine" and start < bp <= end
    if branch_due and not distributed and bp not in schedule:
        milestones += 1  # the serial trainer saves the branch point as a milestone
    keep = retention["keep_recovery_checkpoints"]
    counts = {"initial": int(retention["save_initial_checkpoint"]), "final": 1, "milestones": milestones,
              "separate_90_percent_branch": int(branch_due and distributed),
              # a new recovery checkpoint is staged before the oldest is pruned
              "rolling_recovery_including_staging": min(updates, keep + 1) if keep else 0}

    inv = _inventory(cfg, world, distributed)
    each = _on_disk(inv.tensor_bytes(), world if distributed else 1)
    export = _on_disk(inv.portable_parameters + inv.unique_buffers, 1) if export_weights else 0
    total_count = sum(counts.values())
    return {"kind": "checkpoint_storage_projection", "required_additional_bytes": each * total_count + export,
            "per_checkpoint_estimate_bytes": each, "export_weights_estimate_bytes": export,
            "checkpoint_count": total_count, "count_breakdown": counts, "milestone_policy": schedule.policy(),
            "checkpoint_retention_policy": retention, "start_tokens": start, "token_limit": limit,
            "reachable_tokens": reachable, "reachable_updates": updates, "distributed": distributed,
            "world_size": world, "dtype": str(torch.get_default_dtype()),
            "tensor_bytes_breakdown": {"parameters": inv.parameters, "optimizer_moments": inv.moments,
                                       "optimizer_step_scalars": inv.step_scalars,
                                       "persistent_buffers": inv.buffers,
                                       "distributed_shard_padding_allowance": inv.padding},
            "metadata_allowance_bytes_per_rank_checkpoint": METADATA_ALLOWANCE,
            "scope": "advisory projection, not guaranteed upper bound; no reservation or deletion"}
