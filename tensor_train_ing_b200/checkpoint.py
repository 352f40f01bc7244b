"""Atomic, immutable full-state checkpoints: ``<dir>/state.pt`` + ``<dir>/manifest.json``.

The on-disk format is the reference's (tnlm/checkpoint.py:113-291, format_version 1), so
checkpoints move between the two frameworks in both directions:

* ``state.pt``: a torch pickle ``{format_version, model, model_class, optimizer_class, optimizer,
  sampler, scheduler, scaler, rng, config, progress, manifest_hash, parent, extra, code,
  environment}``;
* ``manifest.json``: ``{format_version, created_utc, files: {state.pt: {sha256, bytes}},
  data_manifest_hash, parent, disk_admission}``.

Saving refuses non-finite tensors and half-collected norm statistics (a checkpoint sits on an
optimizer-step boundary), reserves disk space, writes both files into a staging directory beside
the destination and publishes it with a no-replace rename.  Loading is split in two: a preflight
that checks the files' size and sha256, the payload's identity (format, parent, data manifest,
config) and its compatibility with the live objects (model keys and shapes, optimizer class and
group layout, RNG device count) without touching them, then the restore.  A failed preflight
leaves model, optimizer and sampler as they were.  Load only trusted files: torch pickles can
execute code.
"""
from __future__ import annotations

import dataclasses
import importlib.metadata
import json
import os
import platform
import random
import shutil
import subprocess
import sys
import tempfile
from datetime import datetime, timezone
from pathlib import Path

import numpy as np
import torch

from .checkpoint_storage import checkpoint_space_estimate, require_checkpoint_space
from .durable import fsync_dir, publish_dir
from .hashing import file_sha256

FORMAT_VERSION = 1
PACKAGE = Path(__file__).resolve().parent
_SOURCE_SUFFIXES = (".py", ".cu", ".cuh", ".h", ".cpp")
_STATISTIC_BUFFERS = ("acc_count", "acc_sum")  # lagged-norm accumulators, non-zero mid-update
_RESTORABLE = ("optimizer", "sampler", "scheduler", "scaler")


# ====================================================================================== shared pieces
def to_plain(value):
    """``value`` with dataclasses, tuples and paths turned into dicts, lists and strings."""
    if dataclasses.is_dataclass(value):
        value = dataclasses.asdict(value)
    if isinstance(value, dict):
        return {str(k): to_plain(v) for k, v in value.items()}
    if isinstance(value, (tuple, list)):
        return [to_plain(v) for v in value]
    return str(value) if isinstance(value, Path) else value


def assert_finite(value, where: str):
    """ValueError naming the first floating tensor inside ``value`` that holds a NaN or inf."""
    stack = [(value, where)]
    while stack:
        item, path = stack.pop()
        if isinstance(item, torch.Tensor):
            if (item.is_floating_point() or item.is_complex()) and not bool(torch.isfinite(item).all()):
                raise ValueError(f"Nonfinite checkpoint tensor: {path}")
        elif isinstance(item, dict):
            stack += [(v, f"{path}.{k}") for k, v in reversed(list(item.items()))]
        elif isinstance(item, (list, tuple)):
            stack += [(v, f"{path}[{i}]") for i, v in reversed(list(enumerate(item)))]


def code_identity() -> dict:
    """Git revision, dirtiness and a sha256 of every source file of the package."""
    def git(*args):
        done = subprocess.run(["git", *args], cwd=PACKAGE, capture_output=True, text=True)
        return done.stdout.strip() if done.returncode == 0 else None
    status = git("status", "--porcelain")
    sources = sorted(p for p in PACKAGE.rglob("*") if p.suffix in _SOURCE_SUFFIXES and p.is_file())
    return {"revision": git("rev-parse", "HEAD"), "dirty": None if status is None else bool(status),
            "source_sha256": {f"{PACKAGE.name}/{p.relative_to(PACKAGE).as_posix()}": file_sha256(p) for p in sources}}


def rng_capture() -> dict:
    return {"python": random.getstate(), "numpy": np.random.get_state(), "torch": torch.get_rng_state(),
            "cuda": torch.cuda.get_rng_state_all() if torch.cuda.is_available() else None}


def rng_check(state: dict):
    """The saved generator states can be restored here (same CUDA device count)."""
    if state["cuda"] is None:
        return
    if not torch.cuda.is_available():
        raise ValueError("Checkpoint has CUDA RNG state but CUDA is unavailable")
    if len(state["cuda"]) != torch.cuda.device_count():
        raise ValueError("CUDA device count differs from checkpoint")


def rng_restore(state: dict):
    rng_check(state)
    random.setstate(state["python"])
    np.random.set_state(state["numpy"])
    torch.set_rng_state(state["torch"].cpu())
    if state["cuda"] is not None:
        torch.cuda.set_rng_state_all([s.cpu() for s in state["cuda"]])


def _environment() -> dict:
    cuda_devices = [{"name": torch.cuda.get_device_name(i), "capability": list(torch.cuda.get_device_capability(i))}
                    for i in range(torch.cuda.device_count())]
    packages = sorted((d.metadata["Name"], d.version) for d in importlib.metadata.distributions() if d.metadata["Name"])
    return {"python": sys.version, "platform": platform.platform(), "distributions": dict(packages),
            "torch": str(torch.__version__), "numpy": np.__version__, "cuda": torch.version.cuda,
            "cudnn": torch.backends.cudnn.version(), "torch_build": torch.__config__.show(), "devices": cuda_devices,
            "deterministic_algorithms": torch.are_deterministic_algorithms_enabled(),
            "deterministic_warn_only": torch.is_deterministic_algorithms_warn_only_enabled(),
            "cudnn_deterministic": torch.backends.cudnn.deterministic,
            "cudnn_benchmark": torch.backends.cudnn.benchmark,
            "cuda_matmul_allow_tf32": torch.backends.cuda.matmul.allow_tf32,
            "cudnn_allow_tf32": torch.backends.cudnn.allow_tf32,
            "float32_matmul_precision": torch.get_float32_matmul_precision(),
            "kernel_revision": os.environ.get("TNLM_KERNEL_REVISION")}


def _class_name(obj) -> str:
    return f"{type(obj).__module__}.{type(obj).__qualname__}"


def _durable_json(path: Path, value):
    with path.open("w") as fh:
        json.dump(value, fh, sort_keys=True, indent=2)
        fh.write("\n")
        fh.flush()
        os.fsync(fh.fileno())


# ====================================================================================== saving
def _pending_statistics(model) -> str | None:
    for name, module in model.named_modules():
        for buf in _STATISTIC_BUFFERS:
            value = getattr(module, buf, None)
            if value is not None and bool(torch.as_tensor(value).ne(0).any()):
                return f"{name}.{buf}"
    return None


def save_checkpoint(path, model, optimizer, sampler, *, config, progress, manifest_hash, scheduler=None,
                    scaler=None, parent=None, extra=None) -> dict:
    """Write a new immutable checkpoint directory; returns its manifest."""
    assert_finite(model.state_dict(), "model")
    if optimizer is not None:
        assert_finite(optimizer.state_dict(), "optimizer")
    pending = _pending_statistics(model)
    if pending is not None:
        raise ValueError(f"Checkpoint requires an optimizer-step boundary: {pending} has unfinished statistic collection")
    path = Path(path)
    if path.exists():
        raise FileExistsError(f"Checkpoint already exists: {path}")
    optimizer_class = None
    if optimizer is not None:
        optimizer_class = getattr(optimizer, "checkpoint_class", None) or _class_name(optimizer)
    state = {"format_version": FORMAT_VERSION, "model": model.state_dict(), "model_class": _class_name(model),
             "optimizer_class": optimizer_class,
             **{name: obj.state_dict() if obj is not None else None
                for name, obj in zip(_RESTORABLE, (optimizer, sampler, scheduler, scaler))},
             "rng": rng_capture(), "config": to_plain(config), "progress": to_plain(progress),
             "manifest_hash": manifest_hash, "parent": to_plain(parent), "extra": extra,
             "code": code_identity(), "environment": _environment()}
    admission = require_checkpoint_space(path.parent, checkpoint_space_estimate(
        {"payload": state, "manifest": {"data_manifest_hash": manifest_hash, "parent": to_plain(parent)}}))
    path.parent.mkdir(parents=True, exist_ok=True)
    staging = Path(tempfile.mkdtemp(prefix=f".{path.name}.tmp-", dir=path.parent))
    try:
        state_file = staging / "state.pt"
        with state_file.open("wb") as fh:
            torch.save(state, fh)
            fh.flush()
            os.fsync(fh.fileno())
        manifest = {"format_version": FORMAT_VERSION, "created_utc": datetime.now(timezone.utc).isoformat(),
                    "files": {"state.pt": {"sha256": file_sha256(state_file), "bytes": state_file.stat().st_size}},
                    "data_manifest_hash": manifest_hash, "parent": to_plain(parent), "disk_admission": admission}
        _durable_json(staging / "manifest.json", manifest)
        fsync_dir(staging)
        publish_dir(staging, path)
        return manifest
    finally:
        if staging.exists():
            shutil.rmtree(staging)


# ====================================================================================== reading
def _is_sha256(text) -> bool:
    return isinstance(text, str) and len(text) == 64 and set(text) <= set("0123456789abcdef")


def read_manifest(path) -> dict:
    """The checkpoint's manifest, after checking that it is complete and of this format."""
    path = Path(path)
    try:
        manifest = json.loads((path / "manifest.json").read_text())
        entry = manifest["files"]["state.pt"]
        if not (_is_sha256(entry["sha256"]) and type(entry["bytes"]) is int and entry["bytes"] > 0
                and "data_manifest_hash" in manifest):
            raise ValueError("invalid state checksum metadata")
    except (OSError, ValueError, KeyError, TypeError) as e:
        raise ValueError(f"Incomplete or invalid checkpoint: {path}") from e
    if manifest.get("format_version") != FORMAT_VERSION:
        raise ValueError("Unsupported checkpoint format")
    return manifest


def verified_state_path(path) -> Path:
    """Path to state.pt after checking its size and sha256 against the manifest."""
    entry = read_manifest(path)["files"]["state.pt"]
    state = Path(path) / "state.pt"
    if not state.is_file() or state.stat().st_size != entry["bytes"] or file_sha256(state) != entry["sha256"]:
        raise ValueError("Checkpoint state checksum/size mismatch")
    return state


def _same_optimizer(saved_class, optimizer) -> bool:
    """Optimizer identity: the recorded class is this optimizer's checkpoint class or its own
    class; the reference's and this package's class of the same optimizer count as one."""
    if saved_class is None or saved_class in (getattr(optimizer, "checkpoint_class", None), _class_name(optimizer)):
        return True
    return saved_class.rsplit(".", 1)[-1] == type(optimizer).__qualname__


def _check_optimizer_layout(optimizer, saved):
    """Same number of groups and of parameters per group (the Muon+AdamW pair recursively)."""
    if isinstance(saved, dict) and "param_groups" in saved:
        groups = saved["param_groups"]
        sizes = [len(g.get("params", [])) for g in groups]
        if sizes != [len(g["params"]) for g in optimizer.param_groups]:
            raise ValueError("Checkpoint optimizer parameter groups mismatch")
        return
    pair = isinstance(saved, dict) and set(saved) == {"muon", "adamw"}
    if not pair or not all(isinstance(getattr(optimizer, n, None), torch.optim.Optimizer) for n in saved):
        raise ValueError("Checkpoint optimizer state layout mismatch")
    for name, part in saved.items():
        _check_optimizer_layout(getattr(optimizer, name), part)


class _Preflight:
    """Every check of a loaded payload against its manifest, the caller's expectations and the
    live objects; nothing here modifies those objects."""

    def __init__(self, payload, manifest, targets):
        self.payload, self.manifest, self.targets = payload, manifest, targets

    def identity(self, expected_manifest_hash, expected_config, config_validator):
        p, m = self.payload, self.manifest
        if p.get("format_version") != FORMAT_VERSION:
            raise ValueError("Unsupported checkpoint state format")
        if p.get("parent") != m.get("parent"):
            raise ValueError("Checkpoint parent identity is inconsistent")
        if p["manifest_hash"] != m["data_manifest_hash"]:
            raise ValueError("Checkpoint data identity is inconsistent")
        if expected_manifest_hash is not None and p["manifest_hash"] != expected_manifest_hash:
            raise ValueError("Data manifest hash mismatch")
        if expected_config is not None and p["config"] != to_plain(expected_config):
            raise ValueError("Checkpoint config mismatch")
        if config_validator is not None:
            compatibility = config_validator(p["config"])
            if compatibility is not None:
                p["config_compatibility"] = compatibility

    def completeness(self):
        for name, obj in self.targets.items():
            if obj is not None and self.payload[name] is None:
                raise ValueError(f"Checkpoint is missing {name} state")
        assert_finite(self.payload["model"], "model")
        assert_finite(self.payload["optimizer"], "optimizer")

    def model(self, model):
        live, saved = model.state_dict(), self.payload["model"]
        if live.keys() != saved.keys():
            raise ValueError("Checkpoint model keys/buffers mismatch")
        for name, value in live.items():
            other = saved[name]
            if isinstance(value, torch.Tensor) and (not isinstance(other, torch.Tensor) or other.shape != value.shape):
                raise ValueError(f"Checkpoint model shape mismatch: {name}")

    def optimizer(self):
        optimizer = self.targets["optimizer"]
        if optimizer is None:
            return
        if not _same_optimizer(self.payload.get("optimizer_class"), optimizer):
            raise ValueError("Checkpoint optimizer class mismatch")
        _check_optimizer_layout(optimizer, self.payload["optimizer"])


def load_checkpoint(path, model, optimizer=None, sampler=None, *, expected_manifest_hash=None, expected_config=None,
                    scheduler=None, scaler=None, restore_rng=True, map_location="cpu", config_validator=None) -> dict:
    """Verify and restore a trusted local checkpoint; returns the full payload."""
    manifest = read_manifest(path)
    payload = torch.load(verified_state_path(path), map_location=map_location, weights_only=False)
    targets = dict(zip(_RESTORABLE, (optimizer, sampler, scheduler, scaler)))
    check = _Preflight(payload, manifest, targets)
    check.identity(expected_manifest_hash, expected_config, config_validator)
    check.completeness()
    check.model(model)
    check.optimizer()
    if restore_rng:
        rng_check(payload["rng"])
    # restore
    model.load_state_dict(payload["model"], strict=True)
    for name, obj in targets.items():
        if obj is not None:
            obj.load_state_dict(payload[name])
    with torch.no_grad():  # statistics of an abandoned accumulation are discarded
        for module in model.modules():
            for buf in _STATISTIC_BUFFERS:
                value = getattr(module, buf, None)
                if isinstance(value, torch.Tensor):
                    value.zero_()
    if restore_rng:
        rng_restore(payload["rng"])
    return payload
