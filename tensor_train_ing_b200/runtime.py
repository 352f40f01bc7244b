"""Run identity, seeding, parent-config compatibility and the deterministic-execution scope.

Behaviour matches the reference (tnlm/runtime.py:12-227):

* identity: a checkpoint records the full config (every raw section plus the resolved model and
  train dataclasses, the spend-ledger path made absolute, the determinism and stability policy
  resolved) and a child run compares against it;
* compatibility: a resume may raise the token horizon (not under a cosine schedule or TaperNorm,
  whose schedules depend on it) and change ``project`` execution settings except the ledger; a
  context fork may only increase the context; an evaluation additionally pins the whole train
  section.  A field absent from an older checkpoint is read as its dataclass default, but only if
  the current run uses that default;
* determinism: ``train.deterministic`` scopes torch's deterministic-algorithm flags and the cuBLAS
  workspace setting to one training call; once CUDA has created its handles the workspace setting
  is left as it was set.
"""
from __future__ import annotations

import copy
import os
import random
from contextlib import ExitStack, contextmanager
from dataclasses import MISSING, fields
from functools import lru_cache, wraps
from pathlib import Path

import numpy as np
import torch

from .config import Config, ModelConfig, TrainConfig

DETERMINISTIC_CUBLAS = (":4096:8", ":16:8")
DEFAULT_LEDGER = "runs/spend.json"


# ====================================================================================== identity
def deterministic_requested(cfg) -> bool:
    value = getattr(cfg.train, "deterministic", False)
    if type(value) is not bool:
        raise ValueError("train.deterministic must be Boolean")
    return value


def _ledger_path(project: dict) -> Path:
    return Path(project.get("spend_ledger", DEFAULT_LEDGER)).resolve()


def full_config(cfg) -> dict:
    """A run's identity: raw sections overlaid with the resolved model/train sections."""
    from .training_stability import StabilityPolicy
    policy = StabilityPolicy.from_config(cfg)
    identity = {**cfg.raw, **cfg.to_dict()}
    identity["project"] = {**identity.get("project", {}), "spend_ledger": str(_ledger_path(identity.get("project", {})))}
    identity["train"].update(deterministic=deterministic_requested(cfg), stability_every_steps=policy.stability_every,
                             qk_clip_tau=policy.clip_tau, qk_clip_every_steps=policy.clip_every,
                             qk_clip_source=policy.clip_source)
    return identity


def seed_all(seed: int):
    """Seed Python, NumPy and torch (every CUDA device too)."""
    random.seed(seed)
    np.random.seed(seed)
    torch.manual_seed(seed)
    if torch.cuda.is_available():
        torch.cuda.manual_seed_all(seed)


# ====================================================================================== compatibility
# train fields that older checkpoints may lack although the runtime always honoured them (off)
_ALWAYS_SUPPORTED_TRAIN = {"deterministic": False, "stability_every_steps": 0, "qk_clip_tau": 0.0,
                           "qk_clip_every_steps": 0, "qk_clip_source": "probe"}


@lru_cache(maxsize=None)
def _schema_defaults(section: str) -> tuple:
    """(field, default) pairs of a config section's dataclass (factory defaults built fresh)."""
    schema = {"model": ModelConfig, "train": TrainConfig}[section]
    pairs = {}
    for f in fields(schema):
        if f.default is not MISSING:
            pairs[f.name] = f.default
        elif f.default_factory is not MISSING:
            pairs[f.name] = f.default_factory()
    if section == "train":
        for name, value in _ALWAYS_SUPPORTED_TRAIN.items():
            pairs.setdefault(name, value)
    return tuple(pairs.items())


def _default_missing_config(saved: dict, expected: dict):
    """A copy of ``saved`` with absent model/train fields filled with their defaults, allowed only
    where ``expected`` holds exactly that default.  Returns (copy, compatibility record); the
    checkpoint's own record is never rewritten."""
    resolved = copy.deepcopy(saved)
    filled = {}
    for section in ("model", "train"):
        recorded = resolved.get(section)
        if not isinstance(recorded, dict):
            raise ValueError(f"resume config mismatch: missing {section} section")
        wanted = expected.get(section, {})
        for name, default in _schema_defaults(section):
            if name in recorded or name not in wanted:
                continue
            if type(wanted[name]) is not type(default) or wanted[name] != default:
                raise ValueError(f"resume config mismatch: absent {section}.{name} requires its dataclass default")
            recorded[name] = copy.deepcopy(default)
            filled[f"{section}.{name}"] = copy.deepcopy(default)
    return resolved, {"rule": "missing dataclass field requires current default", "defaulted_fields": filled}


def _context_of(identity: dict):
    return identity.get("data", {}).get("context", 512)


def _differences(a, b, prefix="") -> list[str]:
    """Dotted paths at which two nested dicts differ."""
    if not (isinstance(a, dict) and isinstance(b, dict)):
        return [] if a == b else [prefix or "<root>"]
    out = []
    for key in sorted(set(a) | set(b), key=str):
        path = f"{prefix}.{key}" if prefix else str(key)
        if key not in a or key not in b:
            out.append(path)
        else:
            out += _differences(a[key], b[key], path)
    return out


class ParentConfigCheck:
    """Compares a parent checkpoint's recorded config with the config a child run asks for."""

    def __init__(self, cfg, *, context_fork: bool = False):
        if type(context_fork) is not bool:
            raise ValueError("context_fork must be bool")
        self.expected = full_config(cfg)
        self.context_fork = context_fork

    def _align_context(self, parent: dict, child: dict):
        if not self.context_fork:
            return
        old, new = _context_of(parent), _context_of(child)
        if type(old) is not int or type(new) is not int or old <= 0 or new <= old:
            raise ValueError("context fork requires a strictly increasing positive integer context")
        for side in (parent, child):
            side.setdefault("data", {})["context"] = new

    @staticmethod
    def _split_execution(parent: dict, child: dict):
        """Drop the ``project`` sections (execution settings), which may differ but for the ledger."""
        if _ledger_path(parent.pop("project", {})) != _ledger_path(child.pop("project", {})):
            raise ValueError("resume must retain the project spend ledger")

    @staticmethod
    def _check_horizon(parent: dict, child: dict):
        before = parent["train"].pop("rung_total_tokens")
        after = child["train"].pop("rung_total_tokens")
        if after == before:
            return
        if "cosine" in (parent["train"].get("schedule"), child["train"].get("schedule")):
            raise ValueError("cosine resume must retain the exact original token horizon")
        if any(side.get("model", {}).get(f) == "taper" for side in (parent, child)
               for f in ("normalization", "final_normalization")):
            raise ValueError("TaperNorm resume must retain the exact original token horizon")
        if after < before:
            raise ValueError("resume config mismatch: the token horizon may only be promoted upwards")

    def __call__(self, saved: dict) -> dict:
        child = copy.deepcopy(self.expected)
        parent, record = _default_missing_config(saved, child)
        self._align_context(parent, child)
        self._split_execution(parent, child)
        for side in (parent, child):
            side["train"].setdefault("deterministic", False)
        self._check_horizon(parent, child)
        changed = _differences(parent, child)
        if changed:
            raise ValueError("resume config mismatch: only upward token promotion and project execution settings "
                             f"may change (differs: {', '.join(changed[:8])})")
        return record


def resume_validator(cfg, *, context_fork: bool = False):
    """The check a parent checkpoint's config must pass for a resume (or a context fork)."""
    return ParentConfigCheck(cfg, context_fork=context_fork)


def evaluation_validator(cfg):
    """The resume check plus an identical train section (an evaluation pins training identity)."""
    resume_check = ParentConfigCheck(cfg)
    pinned = {**full_config(cfg)["train"]}
    pinned.setdefault("deterministic", False)

    def validate(saved: dict) -> dict:
        record = resume_check(saved)
        recorded = _default_missing_config(saved, full_config(cfg))[0]["train"]
        recorded.setdefault("deterministic", False)
        if recorded != pinned:
            raise ValueError("evaluation config mismatch: checkpoint training identity is pinned")
        return record

    return validate


def record_context_fork(progress: dict, *, old_context, new_context, parent, source_state):
    """Append a context increase, bound to the restored sampler watermark, to the run's progress."""
    history = copy.deepcopy(progress.get("context_history"))
    if history is None:  # a parent from before context histories were recorded
        history = [{"context": old_context, "start_tokens": None, "start_step": None, "source": "legacy_unknown"}]
    history.append({"context": new_context, "start_tokens": progress["tokens"], "start_step": progress["steps"],
                    "source": "context_fork", "parent": copy.deepcopy(parent),
                    "source_sampler": copy.deepcopy(source_state)})
    progress["context_history"] = history
    progress.setdefault("context_fork_exposure", {"prefix_tokens_at_or_before_watermark": 0,
                                                  "masked_prediction_targets": 0})


# ====================================================================================== determinism
def determinism_metadata() -> dict:
    return {"algorithms_enabled": torch.are_deterministic_algorithms_enabled(),
            "warn_only": torch.is_deterministic_algorithms_warn_only_enabled(),
            "cublas_workspace_config": os.environ.get("CUBLAS_WORKSPACE_CONFIG"),
            "cudnn_benchmark": torch.backends.cudnn.benchmark,
            "cudnn_deterministic": torch.backends.cudnn.deterministic,
            "scope": "PyTorch deterministic policy; this framework's sm_100a kernels reduce in a fixed "
                     "order (run-to-run bitwise identical), cross-platform replay needs separate checks"}


class _DeterminismFlags:
    """A snapshot of the process-wide flags the deterministic scope changes."""

    def __init__(self):
        self.meta = determinism_metadata()

    @property
    def cublas_ok(self) -> bool:
        return self.meta["cublas_workspace_config"] in DETERMINISTIC_CUBLAS

    def restore(self, *, keep_cublas: bool):
        torch.use_deterministic_algorithms(self.meta["algorithms_enabled"], warn_only=self.meta["warn_only"])
        torch.backends.cudnn.benchmark = self.meta["cudnn_benchmark"]
        torch.backends.cudnn.deterministic = self.meta["cudnn_deterministic"]
        if keep_cublas:  # cuBLAS handles were created under the current setting
            return
        if self.meta["cublas_workspace_config"] is None:
            os.environ.pop("CUBLAS_WORKSPACE_CONFIG", None)
        else:
            os.environ["CUBLAS_WORKSPACE_CONFIG"] = self.meta["cublas_workspace_config"]


@contextmanager
def deterministic_execution(enabled: bool, *, device):
    """Turn torch's deterministic algorithms on (``enabled``) or off for the body, then restore."""
    if type(enabled) is not bool:
        raise ValueError("train.deterministic must be Boolean")
    saved = _DeterminismFlags()
    cuda_live = torch.device(device).type == "cuda" and torch.cuda.is_initialized()
    if enabled and cuda_live and not saved.cublas_ok:
        raise RuntimeError("deterministic CUDA requires CUBLAS_WORKSPACE_CONFIG=:4096:8 before CUDA initialization; "
                           "launch a fresh process")
    try:
        if enabled:
            if not saved.cublas_ok:
                os.environ["CUBLAS_WORKSPACE_CONFIG"] = ":4096:8"
            torch.backends.cudnn.benchmark = False
            torch.backends.cudnn.deterministic = True
        torch.use_deterministic_algorithms(enabled, warn_only=False)
        yield
    finally:
        saved.restore(keep_cublas=enabled and cuda_live)


def _local_phase(_name, call):
    return call()


def training_execution(*, collective: bool = False, default_device: str = "cuda"):
    """Decorator of the training entry points: load the config if given a path and scope the
    determinism policy to the call (a dry run changes no global state).  ``collective`` passes the
    setup steps through the distributed checkpoint layer's ``_phase`` (a local failure becomes an
    error on every rank)."""

    def decorate(function):
        @wraps(function)
        def wrapped(cfg, *args, **kwargs):
            if collective:
                from .distributed_checkpoint import _phase as phase
            else:
                phase = _local_phase
            cfg = phase("determinism configuration load",
                        lambda: Config.from_yaml(str(cfg)) if isinstance(cfg, (str, Path)) else cfg)
            enabled = phase("determinism validation", lambda: deterministic_requested(cfg))
            if cfg.raw.get("project", {}).get("dry_run", True):
                return function(cfg, *args, **kwargs)
            with ExitStack() as stack:
                phase("determinism setup", lambda: stack.enter_context(
                    deterministic_execution(enabled, device=kwargs.get("device", default_device))))
                return function(cfg, *args, **kwargs)
        return wrapped

    return decorate
