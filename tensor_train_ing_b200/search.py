"""Deterministic planning of an explicit candidate sweep, without launching or reserving runs
(reference tnlm/search.py:33-98)."""
from __future__ import annotations

import copy
import hashlib
import json
import math
import re
from collections.abc import Mapping

from .config import Config, ModelConfig, TrainConfig
from .runtime import full_config
from .train import plan_search

_ALLOWED = {"model", "train", "project", "data", "evaluation"}
_NAME = re.compile(r"[A-Za-z0-9][A-Za-z0-9_.-]{0,127}\Z")


def merge_overrides(base, override):
    """Deep merge of a mapping of overrides into a configuration mapping (mappings merge, scalars replace)."""
    out = copy.deepcopy(base)
    for key, value in override.items():
        if not isinstance(key, str):
            raise ValueError("override keys must be strings")
        if isinstance(value, Mapping):
            if key in out and not isinstance(out[key], Mapping):
                raise ValueError(f"cannot merge mapping into scalar field {key}")
            out[key] = merge_overrides(out.get(key, {}), value)
        else:
            out[key] = copy.deepcopy(value)
    return out


def plan_sweep(base_cfg, candidates) -> dict:
    """Resolve an ordered list of ``{name, overrides}`` candidates into frozen configurations with
    their cost, time and checkpoint-storage projections (fresh, uncooled full-rung trajectories)."""
    if not isinstance(candidates, list) or not candidates:
        raise ValueError("candidates must be a nonempty list")
    base = full_config(base_cfg)
    names, runs = set(), []
    cost = seconds = 0.0
    unpriced, untimed, storage = [], [], 0
    for cand in candidates:
        if not isinstance(cand, Mapping) or set(cand) != {"name", "overrides"}:
            raise ValueError("each candidate requires exactly name and overrides")
        name = cand["name"]
        if not isinstance(name, str) or not _NAME.fullmatch(name) or name in (".", ".."):
            raise ValueError("candidate name must be a safe path component")
        if name in names:
            raise ValueError("candidate names must be unique")
        names.add(name)
        override = cand["overrides"]
        if not isinstance(override, Mapping) or set(override) - _ALLOWED:
            raise ValueError("unknown top-level override keys or nonmapping overrides")
        if any(not isinstance(v, Mapping) for v in override.values()):
            raise ValueError("top-level configuration overrides must be mappings")
        resolved = merge_overrides(base, override)
        try:
            cfg = Config(model=ModelConfig(**resolved["model"]), train=TrainConfig(**resolved["train"]), raw=resolved)
            config = full_config(cfg)
            encoded = json.dumps(config, sort_keys=True, separators=(",", ":"), allow_nan=False)
            plan = plan_search(cfg)
        except (TypeError, AssertionError, OverflowError) as exc:
            raise ValueError(f"invalid candidate configuration: {name}") from exc
        proposed = plan["proposed_runs"]
        if any(r["projected_usd"] is None for r in proposed):
            unpriced.append(name)
        else:
            cost += sum(r["projected_usd"] for r in proposed)
        if any(r["projected_seconds"] is None for r in proposed):
            untimed.append(name)
        else:
            seconds += sum(r["projected_seconds"] for r in proposed)
        storage += plan["checkpoint_storage_plan"]["required_additional_bytes"]
        runs.append({"name": name, "config": config, "config_sha256": hashlib.sha256(encoded.encode()).hexdigest(),
                     "plan": plan})
    if not math.isfinite(cost) or not math.isfinite(seconds):
        raise ValueError("aggregate projected cost/time must be finite")
    return {"kind": "frozen_explicit_sweep_plan", "runs": runs, "candidate_count": len(runs),
            "required_additional_bytes": storage, "projected_usd": None if unpriced else cost,
            "projected_seconds": None if untimed else seconds, "cost_projection_complete": not unpriced,
            "known_projected_usd": cost, "unpriced_candidates": unpriced, "untimed_candidates": untimed,
            "scope": "fresh uncooled full-rung trajectories; separate cooldown and evaluation excluded; nothing runs"}
