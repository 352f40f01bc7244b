"""Run identity, seeding, resume/evaluation compatibility rules and the deterministic-execution scope.

Behaviour follows the reference (tnlm/runtime.py:12-227): the full config (every raw section plus
resolved model/train) is a checkpoint's identity; a resume may only promote the token horizon
upwards or change ``project`` execution settings; a context fork may only increase the context;
deterministic mode scopes ``torch.use_deterministic_algorithms`` and the cuBLAS workspace setting.
"""
from __future__ import annotations

import copy
import os
import random
from contextlib import ExitStack, contextmanager
from dataclasses import MISSING, fields
from functools import wraps
from pathlib import Path

import numpy as np
import torch

from .config import Config, ModelConfig, TrainConfig

DETERMINISTIC_CUBLAS = (":4096:8", ":16:8")


def deterministic_requested(cfg) -> bool:
    value = getattr(cfg.train, "deterministic", False)
    if type(value) is not bool:
        raise ValueError("train.deterministic must be Boolean")
    return value


def full_config(cfg) -> dict:
    """Identity of a run: raw sections + resolved model/train, spend ledger path made absolute."""
    out = {**cfg.raw, **cfg.to_dict()}
    project = dict(out.get("project", {}))
    project["spend_ledger"] = str(Path(project.get("spend_ledger", "runs/spend.json")).resolve())
    out["project"] = project
    out["train"]["deterministic"] = deterministic_requested(cfg)
    from .training_stability import StabilityPolicy
    policy = StabilityPolicy.from_config(cfg)
    out["train"].update(stability_every_steps=policy.stability_every, qk_clip_tau=policy.clip_tau,
                        qk_clip_every_steps=policy.clip_every, qk_clip_source=policy.clip_source)
    return out


def seed_all(seed: int):
    random.seed(seed)
    np.random.seed(seed)
    torch.manual_seed(seed)
    if torch.cuda.is_available():
        torch.cuda.manual_seed_all(seed)


_LEGACY_TRAIN_DEFAULTS = {"deterministic": False, "stability_every_steps": 0, "qk_clip_tau": 0.0,
                          "qk_clip_every_steps": 0, "qk_clip_source": "probe"}


def _default_missing_config(saved: dict, expected: dict):
    """Fill dataclass fields absent from an older checkpoint's config, but only where the current
    run uses the field's default; recorded values are never rewritten."""
    resolved = copy.deepcopy(saved)
    defaulted = {}
    for section, schema in (("model", ModelConfig), ("train", TrainConfig)):
        values = resolved.get(section)
        if not isinstance(values, dict):
            raise ValueError(f"resume config mismatch: missing {section} section")
        defaults = {}
        for f in fields(schema):
            if f.default is not MISSING:
                defaults[f.name] = f.default
            elif f.default_factory is not MISSING:
                defaults[f.name] = f.default_factory()
        if section == "train":
            for k, v in _LEGACY_TRAIN_DEFAULTS.items():
                defaults.setdefault(k, v)
        for name, default in defaults.items():
            if name in values or name not in expected.get(section, {}):
                continue
            current = expected[section][name]
            if type(current) is not type(default) or current != default:
                raise ValueError(f"resume config mismatch: absent {section}.{name} requires its dataclass default")
            values[name] = copy.deepcopy(default)
            defaulted[f"{section}.{name}"] = copy.deepcopy(default)
    return resolved, {"rule": "missing dataclass field requires current default", "defaulted_fields": defaulted}


def resume_validator(cfg, *, context_fork: bool = False):
    """Validator for a parent checkpoint's config: model/data/math frozen; only upward token
    promotion and project execution settings may change (plus the context, for a fork)."""
    if type(context_fork) is not bool:
        raise ValueError("context_fork must be bool")
    expected = full_config(cfg)

    def validate(saved: dict):
        right = copy.deepcopy(expected)
        left, compatibility = _default_missing_config(saved, right)
        if context_fork:
            old_ctx = left.get("data", {}).get("context", 512)
            new_ctx = right.get("data", {}).get("context", 512)
            if type(old_ctx) is not int or type(new_ctx) is not int or old_ctx <= 0 or new_ctx <= old_ctx:
                raise ValueError("context fork requires a strictly increasing positive integer context")
            left.setdefault("data", {})["context"] = new_ctx
            right.setdefault("data", {})["context"] = new_ctx
        prev_project, cur_project = left.pop("project", {}), right.pop("project", {})
        if (Path(prev_project.get("spend_ledger", "runs/spend.json")).resolve()
                != Path(cur_project.get("spend_ledger", "runs/spend.json")).resolve()):
            raise ValueError("resume must retain the project spend ledger")
        left["train"].setdefault("deterministic", False)
        right["train"].setdefault("deterministic", False)
        previous = left["train"].pop("rung_total_tokens")
        requested = right["train"].pop("rung_total_tokens")
        cosine = "cosine" in (left["train"].get("schedule"), right["train"].get("schedule"))
        if cosine and requested != previous:
            raise ValueError("cosine resume must retain the exact original token horizon")
        taper = any(side.get("model", {}).get(f) == "taper" for side in (left, right)
                    for f in ("normalization", "final_normalization"))
        if taper and requested != previous:
            raise ValueError("TaperNorm resume must retain the exact original token horizon")
        if requested < previous or left != right:
            raise ValueError("resume config mismatch: only upward token promotion and project execution "
                             "settings may change")
        return compatibility

    return validate


def record_context_fork(progress: dict, *, old_context, new_context, parent, source_state):
    """Bind a context increase to the restored sampler watermark in the run's progress record."""
    history = copy.deepcopy(progress.get("context_history"))
    if history is None:
        history = [{"context": old_context, "start_tokens": None, "start_step": None, "source": "legacy_unknown"}]
    history.append({"context": new_context, "start_tokens": progress["tokens"], "start_step": progress["steps"],
                    "source": "context_fork", "parent": copy.deepcopy(parent),
                    "source_sampler": copy.deepcopy(source_state)})
    progress["context_history"] = history
    progress.setdefault("context_fork_exposure", {"prefix_tokens_at_or_before_watermark": 0,
                                                  "masked_prediction_targets": 0})


def evaluation_validator(cfg):
    """Like ``resume_validator`` but the whole training section is pinned as well."""
    compatibility = resume_validator(cfg)
    expected_train = full_config(cfg)["train"]
    expected_train.setdefault("deterministic", False)

    def validate(saved):
        meta = compatibility(saved)
        normalized, _ = _default_missing_config(saved, full_config(cfg))
        saved_train = normalized["train"]
        saved_train.setdefault("deterministic", False)
        if saved_train != expected_train:
            raise ValueError("evaluation config mismatch: checkpoint training identity is pinned")
        return meta

    return validate


def determinism_metadata() -> dict:
    return {"algorithms_enabled": torch.are_deterministic_algorithms_enabled(),
            "warn_only": torch.is_deterministic_algorithms_warn_only_enabled(),
            "cublas_workspace_config": os.environ.get("CUBLAS_WORKSPACE_CONFIG"),
            "cudnn_benchmark": torch.backends.cudnn.benchmark,
            "cudnn_deterministic": torch.backends.cudnn.deterministic,
            "scope": "PyTorch deterministic policy; this framework's sm_100a kernels reduce in a fixed "
                     "order (run-to-run bitwise identical), cross-platform replay needs separate checks"}


@contextmanager
def deterministic_execution(enabled: bool, *, device):
    if type(enabled) is not bool:
        raise ValueError("train.deterministic must be Boolean")
    previous = determinism_metadata()
    cuda = torch.device(device).type == "cuda"
    if enabled and cuda and torch.cuda.is_initialized() and previous["cublas_workspace_config"] not in DETERMINISTIC_CUBLAS:
        raise RuntimeError("deterministic CUDA requires CUBLAS_WORKSPACE_CONFIG=:4096:8 before CUDA initialization; "
                           "launch a fresh process")
    try:
        if enabled:
            if previous["cublas_workspace_config"] not in DETERMINISTIC_CUBLAS:
                os.environ["CUBLAS_WORKSPACE_CONFIG"] = ":4096:8"
            torch.backends.cudnn.benchmark = False
            torch.backends.cudnn.deterministic = True
        torch.use_deterministic_algorithms(enabled, warn_only=False)
        yield
    finally:
        torch.use_deterministic_algorithms(previous["algorithms_enabled"], warn_only=previous["warn_only"])
        torch.backends.cudnn.benchmark = previous["cudnn_benchmark"]
        torch.backends.cudnn.deterministic = previous["cudnn_deterministic"]
        if not (enabled and cuda and torch.cuda.is_initialized()):
            if previous["cublas_workspace_config"] is None:
                os.environ.pop("CUBLAS_WORKSPACE_CONFIG", None)
            else:
                os.environ["CUBLAS_WORKSPACE_CONFIG"] = previous["cublas_workspace_config"]


def training_execution(*, collective: bool = False, default_device: str = "cuda"):
    """Decorator: load the config if given a path and scope the determinism policy to the call
    (dry runs change no global state).  ``collective`` wraps setup in the caller's ``_phase``."""

    def decorate(function):
        @wraps(function)
        def wrapped(cfg, *args, **kwargs):
            if collective:
                from .distributed_checkpoint import _phase
            else:
                _phase = lambda _name, call: call()  # noqa: E731
            cfg = _phase("determinism configuration load",
                         lambda: Config.from_yaml(str(cfg)) if isinstance(cfg, (str, Path)) else cfg)
            enabled = _phase("determinism validation", lambda: deterministic_requested(cfg))
            if cfg.raw.get("project", {}).get("dry_run", True):
                return function(cfg, *args, **kwargs)
            with ExitStack() as stack:
                _phase("determinism setup", lambda: stack.enter_context(
                    deterministic_execution(enabled, device=kwargs.get("device", default_device))))
                return function(cfg, *args, **kwargs)
        return wrapped

    return decorate
