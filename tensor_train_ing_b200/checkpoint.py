"""Atomic, immutable full-state checkpoints: ``<dir>/state.pt`` + ``<dir>/manifest.json``.

The on-disk format is the reference's (tnlm/checkpoint.py:113-291, format_version 1), so
checkpoints move between the two frameworks in both directions:

* ``state.pt``: a torch pickle ``{format_version, model, model_class, optimizer_class, optimizer,
  sampler, scheduler, scaler, rng, config, progress, manifest_hash, parent, extra, code,
  environment}``;
* ``manifest.json``: ``{format_version, created_utc, files: {state.pt: {sha256, bytes}},
  data_manifest_hash, parent, disk_admission}``.

Writes go to a sibling staging directory (fsync'd) that is published with
``renameat2(RENAME_NOREPLACE)``; loads verify size and sha256 before unpickling and validate
keys, shapes and optimizer-group layout before mutating anything.  Load only trusted files:
torch pickles can execute code.
"""
from __future__ import annotations

import ctypes
import dataclasses
import hashlib
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

FORMAT_VERSION = 1
PACKAGE = Path(__file__).resolve().parent


def _plain(value):
    if dataclasses.is_dataclass(value):
        return _plain(dataclasses.asdict(value))
    if isinstance(value, dict):
        return {str(k): _plain(v) for k, v in value.items()}
    if isinstance(value, (tuple, list)):
        return [_plain(v) for v in value]
    if isinstance(value, Path):
        return str(value)
    return value


def _digest(path) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as fh:
        while True:
            block = fh.read(1 << 20)
            if not block:
                break
            h.update(block)
    return h.hexdigest()


def _code_identity() -> dict:
    def git(*args):
        r = subprocess.run(["git", *args], cwd=PACKAGE, capture_output=True, text=True)
        return r.stdout.strip() if r.returncode == 0 else None
    status = git("status", "--porcelain")
    sources = sorted([*PACKAGE.rglob("*.py"), *PACKAGE.rglob("*.cu"), *PACKAGE.rglob("*.cuh"),
                      *PACKAGE.rglob("*.h"), *PACKAGE.rglob("*.cpp")])
    return {"revision": git("rev-parse", "HEAD"), "dirty": None if status is None else bool(status),
            "source_sha256": {f"{PACKAGE.name}/{p.relative_to(PACKAGE).as_posix()}": _digest(p) for p in sources}}


def _rng_state() -> dict:
    return {"python": random.getstate(), "numpy": np.random.get_state(), "torch": torch.get_rng_state(),
            "cuda": torch.cuda.get_rng_state_all() if torch.cuda.is_available() else None}


def _validate_rng(state):
    if state["cuda"] is not None:
        if not torch.cuda.is_available():
            raise ValueError("Checkpoint has CUDA RNG state but CUDA is unavailable")
        if len(state["cuda"]) != torch.cuda.device_count():
            raise ValueError("CUDA device count differs from checkpoint")


def _restore_rng(state):
    _validate_rng(state)
    random.setstate(state["python"])
    np.random.set_state(state["numpy"])
    torch.set_rng_state(state["torch"].cpu())
    if state["cuda"] is not None:
        torch.cuda.set_rng_state_all([s.cpu() for s in state["cuda"]])


def _sync_directory(path):
    fd = os.open(path, os.O_RDONLY | os.O_DIRECTORY)
    try:
        os.fsync(fd)
    finally:
        os.close(fd)


def _publish(staging, path):
    """Atomic no-replace rename (Linux renameat2 with RENAME_NOREPLACE = 1)."""
    libc = ctypes.CDLL(None, use_errno=True)
    fn = libc.renameat2
    fn.argtypes = [ctypes.c_int, ctypes.c_char_p, ctypes.c_int, ctypes.c_char_p, ctypes.c_uint]
    fn.restype = ctypes.c_int
    AT_FDCWD = -100
    if fn(AT_FDCWD, os.fsencode(staging), AT_FDCWD, os.fsencode(path), 1) != 0:
        err = ctypes.get_errno()
        raise OSError(err, os.strerror(err), str(path))


def _require_finite(value, where):
    if isinstance(value, torch.Tensor):
        if (value.is_floating_point() or value.is_complex()) and not bool(torch.isfinite(value).all()):
            raise ValueError(f"Nonfinite checkpoint tensor: {where}")
    elif isinstance(value, dict):
        for k, v in value.items():
            _require_finite(v, f"{where}.{k}")
    elif isinstance(value, (list, tuple)):
        for i, v in enumerate(value):
            _require_finite(v, f"{where}[{i}]")


def _environment() -> dict:
    return {
        "python": sys.version, "platform": platform.platform(),
        "distributions": dict(sorted((d.metadata["Name"], d.version) for d in importlib.metadata.distributions()
                                     if d.metadata["Name"])),
        "torch": str(torch.__version__), "numpy": np.__version__, "cuda": torch.version.cuda,
        "cudnn": torch.backends.cudnn.version(), "torch_build": torch.__config__.show(),
        "devices": [{"name": torch.cuda.get_device_name(i), "capability": list(torch.cuda.get_device_capability(i))}
                    for i in range(torch.cuda.device_count())],
        "deterministic_algorithms": torch.are_deterministic_algorithms_enabled(),
        "deterministic_warn_only": torch.is_deterministic_algorithms_warn_only_enabled(),
        "cudnn_deterministic": torch.backends.cudnn.deterministic,
        "cudnn_benchmark": torch.backends.cudnn.benchmark,
        "cuda_matmul_allow_tf32": torch.backends.cuda.matmul.allow_tf32,
        "cudnn_allow_tf32": torch.backends.cudnn.allow_tf32,
        "float32_matmul_precision": torch.get_float32_matmul_precision(),
        "kernel_revision": os.environ.get("TNLM_KERNEL_REVISION"),
    }


def save_checkpoint(path, model, optimizer, sampler, *, config, progress, manifest_hash, scheduler=None,
                    scaler=None, parent=None, extra=None) -> dict:
    """Write a new immutable checkpoint directory and return its manifest."""
    _require_finite(model.state_dict(), "model")
    if optimizer is not None:
        _require_finite(optimizer.state_dict(), "optimizer")
    for name, module in model.named_modules():
        for buf in ("acc_count", "acc_sum"):
            value = getattr(module, buf, None)
            if value is not None and bool(torch.as_tensor(value).ne(0).any()):
                raise ValueError(f"Checkpoint requires an optimizer-step boundary: {name}.{buf} has unfinished "
                                 "statistic collection")
    path = Path(path)
    if path.exists():
        raise FileExistsError(f"Checkpoint already exists: {path}")
    payload = {
        "format_version": FORMAT_VERSION, "model": model.state_dict(),
        "model_class": f"{type(model).__module__}.{type(model).__qualname__}",
        "optimizer_class": (getattr(optimizer, "checkpoint_class", None)
                            or f"{type(optimizer).__module__}.{type(optimizer).__qualname__}") if optimizer else None,
        "optimizer": optimizer.state_dict() if optimizer is not None else None,
        "sampler": sampler.state_dict() if sampler is not None else None,
        "scheduler": scheduler.state_dict() if scheduler is not None else None,
        "scaler": scaler.state_dict() if scaler is not None else None,
        "rng": _rng_state(), "config": _plain(config), "progress": _plain(progress),
        "manifest_hash": manifest_hash, "parent": _plain(parent), "extra": extra,
        "code": _code_identity(), "environment": _environment(),
    }
    admission = require_checkpoint_space(path.parent, checkpoint_space_estimate(
        {"payload": payload, "manifest": {"data_manifest_hash": manifest_hash, "parent": _plain(parent)}}))
    path.parent.mkdir(parents=True, exist_ok=True)
    staging = Path(tempfile.mkdtemp(prefix=f".{path.name}.tmp-", dir=path.parent))
    try:
        state = staging / "state.pt"
        with state.open("wb") as fh:
            torch.save(payload, fh)
            fh.flush()
            os.fsync(fh.fileno())
        manifest = {"format_version": FORMAT_VERSION, "created_utc": datetime.now(timezone.utc).isoformat(),
                    "files": {"state.pt": {"sha256": _digest(state), "bytes": state.stat().st_size}},
                    "data_manifest_hash": manifest_hash, "parent": _plain(parent), "disk_admission": admission}
        with (staging / "manifest.json").open("w") as fh:
            json.dump(manifest, fh, sort_keys=True, indent=2)
            fh.write("\n")
            fh.flush()
            os.fsync(fh.fileno())
        _sync_directory(staging)
        _publish(staging, path)
        _sync_directory(path.parent)
        return manifest
    finally:
        if staging.exists():
            shutil.rmtree(staging)


def read_manifest(path) -> dict:
    path = Path(path)
    try:
        manifest = json.loads((path / "manifest.json").read_text())
        info = manifest["files"]["state.pt"]
        digest, size = info["sha256"], info["bytes"]
        ok = (isinstance(digest, str) and len(digest) == 64 and all(c in "0123456789abcdef" for c in digest)
              and type(size) is int and size > 0 and "data_manifest_hash" in manifest)
        if not ok:
            raise ValueError("invalid state checksum metadata")
    except (OSError, ValueError, KeyError, TypeError) as e:
        raise ValueError(f"Incomplete or invalid checkpoint: {path}") from e
    if manifest.get("format_version") != FORMAT_VERSION:
        raise ValueError("Unsupported checkpoint format")
    return manifest


def verified_state_path(path) -> Path:
    """Path to state.pt after checking its size and sha256 against the manifest."""
    manifest = read_manifest(path)
    info = manifest["files"]["state.pt"]
    state = Path(path) / "state.pt"
    if not state.is_file() or state.stat().st_size != info["bytes"] or _digest(state) != info["sha256"]:
        raise ValueError("Checkpoint state checksum/size mismatch")
    return state


def _validate_optimizer_layout(optimizer, saved):
    if not isinstance(saved, dict):
        raise ValueError("Checkpoint optimizer state layout mismatch")
    if "param_groups" in saved:
        groups = saved["param_groups"]
        if len(groups) != len(optimizer.param_groups) or any(
                len(s.get("params", [])) != len(a["params"]) for s, a in zip(groups, optimizer.param_groups)):
            raise ValueError("Checkpoint optimizer parameter groups mismatch")
    elif set(saved) == {"muon", "adamw"} and all(
            isinstance(getattr(optimizer, n, None), torch.optim.Optimizer) for n in saved):
        for n, child in saved.items():
            _validate_optimizer_layout(getattr(optimizer, n), child)
    else:
        raise ValueError("Checkpoint optimizer state layout mismatch")


def _optimizer_identity_ok(saved_class, optimizer) -> bool:
    """The optimizer class must match; reference and framework classes of the same optimizer
    (e.g. ``tnlm.optim.MuonAdamW`` / ``tensor_train_ing_b200.optim.MuonAdamW``) are equivalent."""
    if saved_class is None or saved_class == getattr(optimizer, "checkpoint_class", None):
        return True
    ours = f"{type(optimizer).__module__}.{type(optimizer).__qualname__}"
    if saved_class == ours:
        return True
    return saved_class.rsplit(".", 1)[-1] == type(optimizer).__qualname__


def load_checkpoint(path, model, optimizer=None, sampler=None, *, expected_manifest_hash=None, expected_config=None,
                    scheduler=None, scaler=None, restore_rng=True, map_location="cpu", config_validator=None) -> dict:
    """Verify and restore a trusted local checkpoint; returns the full payload."""
    manifest = read_manifest(path)
    state = verified_state_path(path)
    payload = torch.load(state, map_location=map_location, weights_only=False)
    if payload.get("format_version") != FORMAT_VERSION:
        raise ValueError("Unsupported checkpoint state format")
    if payload.get("parent") != manifest.get("parent"):
        raise ValueError("Checkpoint parent identity is inconsistent")
    if payload["manifest_hash"] != manifest["data_manifest_hash"]:
        raise ValueError("Checkpoint data identity is inconsistent")
    if expected_manifest_hash is not None and payload["manifest_hash"] != expected_manifest_hash:
        raise ValueError("Data manifest hash mismatch")
    if expected_config is not None and payload["config"] != _plain(expected_config):
        raise ValueError("Checkpoint config mismatch")
    if config_validator is not None:
        compat = config_validator(payload["config"])
        if compat is not None:
            payload["config_compatibility"] = compat
    for name, obj in (("optimizer", optimizer), ("sampler", sampler), ("scheduler", scheduler), ("scaler", scaler)):
        if obj is not None and payload[name] is None:
            raise ValueError(f"Checkpoint is missing {name} state")
    _require_finite(payload["model"], "model")
    _require_finite(payload["optimizer"], "optimizer")
    current, incoming = model.state_dict(), payload["model"]
    if current.keys() != incoming.keys():
        raise ValueError("Checkpoint model keys/buffers mismatch")
    for name, value in current.items():
        saved = incoming[name]
        if isinstance(value, torch.Tensor) and (not isinstance(saved, torch.Tensor) or value.shape != saved.shape):
            raise ValueError(f"Checkpoint model shape mismatch: {name}")
    if optimizer is not None:
        if not _optimizer_identity_ok(payload.get("optimizer_class"), optimizer):
            raise ValueError("Checkpoint optimizer class mismatch")
        _validate_optimizer_layout(optimizer, payload["optimizer"])
    if restore_rng:
        _validate_rng(payload["rng"])
    model.load_state_dict(incoming, strict=True)
    for name, obj in (("optimizer", optimizer), ("sampler", sampler), ("scheduler", scheduler), ("scaler", scaler)):
        if obj is not None:
            obj.load_state_dict(payload[name])
    for module in model.modules():  # statistics of an abandoned accumulation are discarded
        for name in ("acc_count", "acc_sum"):
            value = getattr(module, name, None)
            if isinstance(value, torch.Tensor):
                with torch.no_grad():
                    value.zero_()
    if restore_rng:
        _restore_rng(payload["rng"])
    return payload
