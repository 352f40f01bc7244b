"""Sharded recovery checkpoints for owner-computes data parallelism (reference
tnlm/distributed_checkpoint.py:46-483, format ``tnlm-dcp-v1``; this framework writes ``ttb-sharded-v1``).

Directory layout (published atomically with a no-replace rename, like the full-state format):

* ``model.pt``        the model state (parameters are replicated between steps; rank 0 writes it);
                      under parameter sharding only the replicated part;
* ``rank-XXXXX.pt``   each rank's optimizer state (only the parameters it owns), RNG states and
                      sampler cursor, and under parameter sharding the fp32 masters it owns;
* ``manifest.json``   format, world size, torch version, backend, the ownership layout, the
                      replicated-buffer digest, config / progress / data identity and the sha256
                      and size of every file.

Exact replay needs the same world size, layout and torch version, as in the reference.  Every
rank must call each function in the same order with a live process group.  ``_phase`` and
``_agree`` are the control-plane helpers the distributed trainer uses: a rank-local exception
becomes an error on every rank instead of a hang in the next collective.
"""
from __future__ import annotations

import hashlib
import json
import os
import shutil
import tempfile
from datetime import datetime, timezone
from pathlib import Path

import torch
import torch.distributed as dist

from .checkpoint import assert_finite, code_identity, rng_capture, rng_check, rng_restore, to_plain
from .durable import fsync_dir, publish_dir
from .hashing import file_sha256
from .checkpoint_storage import checkpoint_space_estimate, require_checkpoint_space

FORMAT = "ttb-sharded-v1"


def _group():
    if not dist.is_initialized():
        raise ValueError("distributed checkpoint requires an initialized process group")
    return dist.get_rank(), dist.get_world_size()


def _phase(label, callback):
    """Run ``callback`` on every rank; if any rank raised, raise on all of them (with every message)."""
    value, error = None, None
    try:
        value = callback()
    except Exception as exc:  # noqa: BLE001 - converted into an all-rank failure
        error = f"{type(exc).__name__}: {exc}"
    errors = [None] * dist.get_world_size()
    dist.all_gather_object(errors, error)
    if any(errors):
        raise ValueError(f"{label} failed: " + "; ".join(f"rank {i}: {e}" for i, e in enumerate(errors) if e))
    return value


def _agree(label, value):
    """Require every rank to hold the same JSON-serialisable value."""
    encoded = _phase(f"{label} serialization", lambda: json.dumps(value, sort_keys=True, allow_nan=False))
    values = [None] * dist.get_world_size()
    dist.all_gather_object(values, encoded)
    if len(set(values)) != 1:
        raise ValueError(f"{label} differs across ranks")
    return value


def _tensor_digest(items) -> str:
    h = hashlib.sha256()
    for name, value in sorted(items):
        value = value.detach().cpu().contiguous()
        h.update(json.dumps([name, str(value.dtype), list(value.shape)]).encode())
        h.update(value.reshape(-1).view(torch.uint8).numpy().tobytes())
    return h.hexdigest()


def _replicated_state(model, dp=None) -> dict:
    """Everything every rank holds identically between steps (all of the model unless its
    parameters are sharded)."""
    if dp is not None and getattr(dp, "shard_params", False):
        return dp.replicated_state()
    return model.state_dict()


def _replicated_digest(model, dp=None) -> str:
    """Digest of everything that must be identical on every rank: parameters and buffers."""
    return _tensor_digest(_replicated_state(model, dp).items())


def _layout(dp, optimizer) -> dict:
    """Ownership layout shared by every rank (this rank's optimizer groups are checked separately)."""
    return {"units": dp.layout, "shard": dp.shard, "world": dp.world,
            "optimizer_class": f"{type(optimizer).__qualname__}"}


def _local_layout(optimizer) -> list:
    return [[list(p.shape) for p in g["params"]] for g in optimizer.param_groups]


def _runtime() -> dict:
    return {"torch": str(torch.__version__), "backend": str(dist.get_backend())}


def _check_boundary(model):
    for name, module in model.named_modules():
        for buf in ("acc_count", "acc_sum"):
            value = getattr(module, buf, None)
            if value is not None and bool(torch.as_tensor(value).ne(0).any()):
                raise ValueError(f"checkpoint requires an optimizer-step boundary: {name}.{buf} is collecting")


def save_distributed_checkpoint(path, model, optimizer, sampler, dp, *, config, progress, manifest_hash,
                                parent=None, extra=None) -> dict:
    """Collectively write a new immutable sharded checkpoint directory; returns its manifest."""
    rank, world = _group()
    path = Path(path).resolve()

    def preflight():
        assert_finite(model.state_dict(), "model")
        assert_finite(optimizer.state_dict(), "optimizer")
        _check_boundary(model)
        if path.exists():
            raise FileExistsError(f"checkpoint already exists: {path}")
        return {"path": str(path), "world_size": world, "layout": _layout(dp, optimizer), "runtime": _runtime(),
                "config": to_plain(config), "progress": to_plain(progress), "manifest_hash": manifest_hash,
                "parent": to_plain(parent), "extra": to_plain(extra)}
    shared = _agree("checkpoint request", _phase("checkpoint preflight", preflight))
    digest = _agree("replicated state", _phase("replicated digest", lambda: _replicated_digest(model, dp)))
    sharded = bool(getattr(dp, "shard_params", False))
    local = {"rank": rank, "world_size": world, "optimizer": optimizer.state_dict(),
             "optimizer_layout": _local_layout(optimizer),
             "sampler": sampler.state_dict() if sampler is not None else None, "rng": rng_capture(),
             "owned_params": ({k: v.cpu() for k, v in dp.owned_sharded_state().items()} if sharded else None)}
    replicated = _replicated_state(model, dp)

    def staging():
        if rank == 0:
            estimate = checkpoint_space_estimate({"local": local, "model": replicated}) * (2 + world * sharded)
            require_checkpoint_space(path.parent, estimate)
            path.parent.mkdir(parents=True, exist_ok=True)
            return tempfile.mkdtemp(prefix=f".{path.name}.tmp-", dir=path.parent)
        return None
    box = [_phase("staging directory", staging)]
    dist.broadcast_object_list(box, src=0)
    stage = Path(box[0])
    try:
        def write():
            out = {}
            name = f"rank-{rank:05d}.pt"
            with (stage / name).open("wb") as fh:
                torch.save(local, fh)
                fh.flush()
                os.fsync(fh.fileno())
            out[name] = {"sha256": file_sha256(stage / name), "bytes": (stage / name).stat().st_size}
            if rank == 0:
                with (stage / "model.pt").open("wb") as fh:
                    torch.save({"model": replicated}, fh)
                    fh.flush()
                    os.fsync(fh.fileno())
                out["model.pt"] = {"sha256": file_sha256(stage / "model.pt"), "bytes": (stage / "model.pt").stat().st_size}
            return out
        files = _phase("rank file write", write)
        gathered = [None] * world
        dist.all_gather_object(gathered, files)

        def publish():
            if rank != 0:
                return None
            manifest = {"format": FORMAT, "created_utc": datetime.now(timezone.utc).isoformat(), **shared,
                        "replicated_state_sha256": digest, "code": code_identity(),
                        "files": {k: v for part in gathered for k, v in part.items()},
                        "replay_scope": "same world size, layout and torch version; rank-local RNG and data cursors"}
            with (stage / "manifest.json").open("w") as fh:
                json.dump(manifest, fh, sort_keys=True, indent=2, allow_nan=False)
                fh.write("\n")
                fh.flush()
                os.fsync(fh.fileno())
            fsync_dir(stage)
            publish_dir(stage, path)
            return manifest
        box = [_phase("atomic publication", publish)]
        dist.broadcast_object_list(box, src=0)
        return box[0]
    finally:
        if rank == 0 and stage.exists():
            shutil.rmtree(stage, ignore_errors=True)


def read_distributed_manifest(path) -> dict:
    manifest = json.loads((Path(path) / "manifest.json").read_text())
    if manifest.get("format") != FORMAT:
        raise ValueError(f"not a {FORMAT} checkpoint")
    return manifest


def is_distributed_checkpoint(path) -> bool:
    try:
        return json.loads((Path(path) / "manifest.json").read_text()).get("format") == FORMAT
    except (OSError, ValueError):
        return False


def load_distributed_checkpoint(path, model, optimizer, sampler, dp, *, expected_manifest_hash=None,
                                config_validator=None, restore_rng=True) -> dict:
    """Verify every file, then restore model, this rank's optimizer shard, sampler and RNG."""
    rank, world = _group()
    path = Path(path).resolve()

    def verify():
        manifest = read_distributed_manifest(path)
        if manifest["world_size"] != world:
            raise ValueError(f"checkpoint world size {manifest['world_size']} != {world}")
        if manifest["runtime"] != _runtime():
            raise ValueError("checkpoint torch version or backend differs")
        if manifest["layout"] != _layout(dp, optimizer):
            raise ValueError("checkpoint ownership/optimizer layout differs")
        if expected_manifest_hash is not None and manifest["manifest_hash"] != expected_manifest_hash:
            raise ValueError("data manifest hash mismatch")
        expected = {f"rank-{i:05d}.pt" for i in range(world)} | {"model.pt"}
        actual = {p.name for p in path.iterdir() if p.is_file()} - {"manifest.json"}
        if set(manifest["files"]) != expected or actual != expected:
            raise ValueError("checkpoint file set differs from manifest")
        for name in ("model.pt", f"rank-{rank:05d}.pt"):
            info = manifest["files"][name]
            if (path / name).stat().st_size != info["bytes"] or file_sha256(path / name) != info["sha256"]:
                raise ValueError(f"checkpoint checksum mismatch: {name}")
        compat = config_validator(manifest["config"]) if config_validator is not None else None
        return manifest, compat
    manifest, compat = _phase("checkpoint verification", verify)
    _agree("checkpoint identity", manifest["replicated_state_sha256"])

    def stage():
        state = torch.load(path / "model.pt", map_location="cpu", weights_only=False)["model"]
        local = torch.load(path / f"rank-{rank:05d}.pt", map_location="cpu", weights_only=False)
        if local["rank"] != rank or local["world_size"] != world:
            raise ValueError("rank file identity mismatch")
        if local["optimizer_layout"] != _local_layout(optimizer):
            raise ValueError("this rank's optimizer parameter layout differs from the checkpoint")
        assert_finite(state, "model")
        assert_finite(local["optimizer"], "optimizer")
        if restore_rng:
            rng_check(local["rng"])
        current = _replicated_state(model, dp)
        if current.keys() != state.keys() or any(current[k].shape != state[k].shape for k in current):
            raise ValueError("checkpoint model keys or shapes differ")
        if getattr(dp, "shard_params", False):
            owned = dp.owned_sharded_state()
            mine = local.get("owned_params") or {}
            if mine.keys() != owned.keys() or any(mine[k].shape != owned[k].shape for k in owned):
                raise ValueError("this rank's sharded parameters differ from the checkpoint")
            assert_finite(mine, "sharded parameters")
        if sampler is not None and local["sampler"] is None:
            raise ValueError("checkpoint has no sampler state")
        return state, local
    state, local = _phase("checkpoint staging", stage)

    def install():
        with torch.no_grad():
            current = _replicated_state(model, dp)
            for k, v in state.items():
                current[k].copy_(v)  # in place: parameters stay views of the flat buffers
            if getattr(dp, "shard_params", False):
                dp.load_owned_sharded(local["owned_params"])
        optimizer.load_state_dict(local["optimizer"])
        if sampler is not None:
            sampler.load_state_dict(local["sampler"])
        if restore_rng:
            rng_restore(local["rng"])
    _phase("checkpoint install", install)
    if getattr(dp, "shard_params", False):
        dp.gather_params()  # bf16 caches / compute copies from the restored masters
    digest = _replicated_digest(model, dp)
    if digest != manifest["replicated_state_sha256"]:
        raise ValueError("restored replicated state digest differs from the manifest")
    out = dict(manifest)
    if compat is not None:
        out["config_compatibility"] = compat
    return out


def export_distributed_weights(path, model, *, config, progress, manifest_hash, parent=None,
                               max_state_bytes=4_000_000_000, dp=None) -> dict:
    """Collectively export the model as a full-state checkpoint for serial evaluators (with
    parameter sharding, ``dp`` assembles the owners' masters on rank 0).

    Only rank 0 writes; the result has no optimizer or sampler state and does not resume training."""
    from .checkpoint import save_checkpoint
    rank, world = _group()
    sharded = bool(getattr(dp, "shard_params", False))

    def preflight():
        if type(max_state_bytes) is not int or max_state_bytes <= 0:
            raise ValueError("positive integer export state-byte limit required")
        _check_boundary(model)
        state = model.state_dict()
        assert_finite(_replicated_state(model, dp), "model")
        size = sum(v.numel() * v.element_size() for v in state.values())
        if size > max_state_bytes:
            raise ValueError(f"full export needs {size} tensor bytes, exceeds {max_state_bytes}")
        if Path(path).exists():
            raise ValueError("export destination already exists")
        return {"path": str(Path(path).resolve()), "state_bytes": size}
    request = _agree("export request", _phase("export preflight", preflight))
    _agree("export replicated state", _replicated_digest(model, dp))
    full = dp.full_state_dict(dst=0) if sharded else None

    def publish():
        if rank:
            return None
        source = model
        if sharded:  # a CPU model holding the assembled state
            with torch.device("meta"):
                source = type(model)(model.cfg)
            source.load_state_dict(full, assign=True)
            assert_finite(full, "model")
        return save_checkpoint(request["path"], source, None, None, config=config, progress=progress,
                               manifest_hash=manifest_hash, parent=parent,
                               extra={"artifact_kind": "distributed_evaluation_weights", "training_recovery": False,
                                      "source_world_size": world, "persistent_tensor_bytes": request["state_bytes"]})
    box = [_phase("evaluation artifact publication", publish)]
    dist.broadcast_object_list(box, src=0)
    return box[0]
