"""Plan an explicit sweep without running anything.

Each candidate's overrides are laid over the base configuration, the result is frozen together with
its canonical sha256, and the per-candidate cost, time and checkpoint-storage projections of
``train.plan_search`` are totalled.  No model runs, no ledger row is reserved and no directory is
created.  The rules are the reference planner's (tnlm/search.py:33-98): a candidate is exactly a
``{"name", "overrides"}`` mapping, names are unique safe path components, overrides name only the
configuration's top-level sections and merge mapping by mapping (a mapping never replaces a scalar).
"""
from __future__ import annotations

import copy
import math
import re
from collections.abc import Mapping
from dataclasses import dataclass, field

from .config import Config, ModelConfig, TrainConfig
from .hashing import canonical_json, text_sha256
from .runtime import full_config
from .train import plan_search

SECTIONS = frozenset({"model", "train", "project", "data", "evaluation"})
_SAFE_NAME = re.compile(r"[A-Za-z0-9][A-Za-z0-9_.-]{0,127}\Z")


def overlay(base: Mapping, patch: Mapping, where: str = "") -> dict:
    """``base`` with ``patch`` laid over it: nested mappings merge key by key, other values replace."""
    merged = copy.deepcopy(dict(base))
    for key, value in patch.items():
        if not isinstance(key, str):
            raise ValueError(f"override keys must be strings (got {key!r} under {where or 'the top level'})")
        path = f"{where}.{key}" if where else key
        if isinstance(value, Mapping):
            if key in merged and not isinstance(merged[key], Mapping):
                raise ValueError(f"override {path} is a mapping but the base value there is not")
            merged[key] = overlay(merged.get(key, {}), value, path)
        else:
            merged[key] = copy.deepcopy(value)
    return merged


def _checked(entry, taken: set) -> tuple[str, Mapping]:
    if not isinstance(entry, Mapping) or set(entry) != {"name", "overrides"}:
        raise ValueError("a sweep candidate is a mapping with exactly the keys name and overrides")
    name, overrides = entry["name"], entry["overrides"]
    if not isinstance(name, str) or name in (".", "..") or not _SAFE_NAME.fullmatch(name):
        raise ValueError(f"candidate name {name!r} is not a safe path component")
    if name in taken:
        raise ValueError(f"candidate name {name!r} is used twice")
    if not isinstance(overrides, Mapping) or not set(overrides) <= SECTIONS:
        raise ValueError(f"candidate {name!r}: overrides must be a mapping of sections among {sorted(SECTIONS)}")
    if not all(isinstance(v, Mapping) for v in overrides.values()):
        raise ValueError(f"candidate {name!r}: each overridden section must be a mapping")
    return name, overrides


@dataclass
class _Totals:
    usd: float = 0.0
    seconds: float = 0.0
    storage: int = 0
    unpriced: list = field(default_factory=list)
    untimed: list = field(default_factory=list)

    def add(self, name: str, plan: dict) -> None:
        runs = plan["proposed_runs"]
        prices = [r["projected_usd"] for r in runs]
        times = [r["projected_seconds"] for r in runs]
        if None in prices:
            self.unpriced.append(name)
        else:
            self.usd += sum(prices)
        if None in times:
            self.untimed.append(name)
        else:
            self.seconds += sum(times)
        self.storage += plan["checkpoint_storage_plan"]["required_additional_bytes"]


def plan_sweep(base_cfg, candidates) -> dict:
    """The frozen plan of an ordered, nonempty candidate list (fresh, uncooled full-rung runs)."""
    if not isinstance(candidates, list) or not candidates:
        raise ValueError("a sweep needs a nonempty list of candidates")
    base = full_config(base_cfg)
    taken: set = set()
    totals = _Totals()
    runs = []
    for entry in candidates:
        name, overrides = _checked(entry, taken)
        taken.add(name)
        resolved = overlay(base, overrides)
        try:
            cfg = Config(model=ModelConfig(**resolved["model"]), train=TrainConfig(**resolved["train"]), raw=resolved)
            frozen = full_config(cfg)
            digest = text_sha256(canonical_json(frozen))
            plan = plan_search(cfg)
        except (TypeError, AssertionError, OverflowError) as exc:
            raise ValueError(f"candidate {name!r} does not resolve to a valid configuration") from exc
        totals.add(name, plan)
        runs.append({"name": name, "config": frozen, "config_sha256": digest, "plan": plan})
    if not (math.isfinite(totals.usd) and math.isfinite(totals.seconds)):
        raise ValueError("the sweep's projected cost or time is not finite")
    return {"kind": "frozen_explicit_sweep_plan", "runs": runs, "candidate_count": len(runs),
            "required_additional_bytes": totals.storage,
            "projected_usd": None if totals.unpriced else totals.usd,
            "projected_seconds": None if totals.untimed else totals.seconds,
            "cost_projection_complete": not totals.unpriced, "known_projected_usd": totals.usd,
            "unpriced_candidates": totals.unpriced, "untimed_candidates": totals.untimed,
            "scope": "fresh full-rung trajectories without cooldown; cooldowns and evaluations not included; "
                     "nothing was run or reserved",
            "storage_scope": "sum of each run's advisory checkpoint projection; existing and pinned artifacts "
                             "not included"}
