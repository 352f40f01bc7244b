"""Interchange with the reference's sharded recovery checkpoints (``tnlm-dcp-v1``).

The reference's distributed trainer saves an FSDP2 job as (tnlm/distributed_checkpoint.py:306-483):

* ``dcp/``: a ``torch.distributed.checkpoint`` directory of ``{"model": ..., "optimizer": ...}``
  whose flattened keys are ``model.<fqn>``, ``optimizer.state.<fqn>.<stat>`` and
  ``optimizer.param_groups.<i>.<key>`` (groups of Muon first, then AdamW, for MuonAdamW);
  the tensors are the logical (unsharded) shapes, stored as the ranks' row shards;
* ``rank-XXXXX.pt``: that rank's RNG states and ``RankPackedSampler`` cursor;
* ``manifest.json``: format, config, progress, data identity, world size, torch version, backend,
  the FSDP2 layout (every state entry's shape, dtype, placement and mesh; the optimizer's parameter
  groups by name), determinism flags, checksums of every file and a digest of the model buffers.

This framework keeps whole parameters on their owning rank (owner-computes) rather than row shards,
so the interchange goes through DCP's resharding: loading requests the logical tensors this rank
needs (all replicated model entries, its owned sharded parameters and the optimizer state of the
parameters it owns) and installs them; saving gives DCP the same logical tensors (replicated entries
from every rank, which DCP writes once; owned ones from their owner) plus the full parameter-group
records, and writes the manifest in the reference's form, with the layout an FSDP2 model of this
world size reports, so the reference's own loader accepts it.  Both directions require the same
world size (the per-rank sampler streams and RNG states are per rank) and, as the reference does,
the same torch version.
"""
from __future__ import annotations

import copy
import json
import os
import shutil
import tempfile
from datetime import datetime, timezone
from pathlib import Path

import torch
import torch.distributed as dist

from .checkpoint import assert_finite, code_identity, rng_capture, rng_check, rng_restore, to_plain
from .checkpoint_storage import checkpoint_space_estimate, require_checkpoint_space
from .distributed_checkpoint import _agree, _phase, _tensor_digest
from .durable import fsync_dir, publish_dir
from .hashing import file_sha256
from .optim import MuonAdamW

FORMAT = "tnlm-dcp-v1"
_REPLAY_SCOPE = "same-world same-layout rank-local RNG/data cursor; group failure requires relaunch"
# group entries that select an implementation rather than the update; written as the reference's
# defaults and never taken from a loaded checkpoint
_IMPLEMENTATION_KEYS = {"fused": None, "foreach": None, "capturable": False, "differentiable": False}
# group entries that define the update; a loaded checkpoint must agree with the live optimizer
_MATH_KEYS = ("betas", "eps", "weight_decay", "momentum", "nesterov", "ns_coefficients", "ns_steps", "adjust_lr_fn",
              "amsgrad", "maximize", "kind")


# ====================================================================================== identity
def _group():
    if not dist.is_initialized():
        raise ValueError("the reference checkpoint format needs an initialized process group")
    return dist.get_rank(), dist.get_world_size()


def _parts(optimizer) -> list:
    """Optimizer children in the order the reference merges their groups."""
    return [optimizer.muon, optimizer.adamw] if isinstance(optimizer, MuonAdamW) else [optimizer]


def _class_path(cls) -> str:
    return f"{cls.__module__}.{cls.__qualname__}"


def _fsdp_model_class(model) -> str:
    """The class name an FSDP2-wrapped model of this type reports (``fully_shard`` builds it as
    ``FSDP<class>`` in its initialisation module)."""
    try:
        from torch.distributed.fsdp._fully_shard import _fsdp_init
        module = _fsdp_init.__name__
    except ImportError:  # an older torch layout
        module = "torch.distributed.fsdp._fully_shard._fully_shard"
    return f"{module}.FSDP{type(model).__name__}"


def _fqns(model) -> dict[int, str]:
    return {id(p): name for name, p in model.named_parameters()}


def _reference_layout(model, logical, world: int, device_type: str) -> dict:
    """The layout the reference's FSDP2 job of ``world`` ranks records for this model/optimizer:
    parameters as ``Shard(0)`` DTensors on a 1-D mesh, buffers as plain tensors."""
    from torch.distributed.tensor import Shard
    params = set(_fqns(model).values())
    mesh = {"shape": [world], "device_type": device_type, "rank_order": list(range(world))}
    entries = {name: {"shape": list(t.shape), "dtype": str(t.dtype),
                      "placements": [str(Shard(0))] if name in params else None,
                      "mesh": copy.deepcopy(mesh) if name in params else None}
               for name, t in model.state_dict().items()}
    names = _fqns(model)
    groups = lambda opt: [[names[id(p)] for p in g["params"]] for g in opt.param_groups]  # noqa: E731
    layout = {"model_class": _fsdp_model_class(model), "model": entries, "optimizer": "torch.optim.AdamW",
              "parameter_groups": groups(logical)}
    if isinstance(logical, MuonAdamW):
        layout["optimizer"] = MuonAdamW.checkpoint_class
        layout["optimizer_children"] = [{"class": _class_path(torch.optim.Muon), "parameter_groups": groups(logical.muon)},
                                        {"class": _class_path(torch.optim.AdamW), "parameter_groups": groups(logical.adamw)}]
    return layout


def _runtime_flags() -> dict:
    return {"deterministic_algorithms": torch.are_deterministic_algorithms_enabled(),
            "deterministic_warn_only": torch.is_deterministic_algorithms_warn_only_enabled(),
            "cudnn_deterministic": torch.backends.cudnn.deterministic,
            "cudnn_benchmark": torch.backends.cudnn.benchmark,
            "cuda_matmul_allow_tf32": torch.backends.cuda.matmul.allow_tf32,
            "cudnn_allow_tf32": torch.backends.cudnn.allow_tf32,
            "float32_matmul_precision": torch.get_float32_matmul_precision()}


def _buffer_digest(model) -> str:
    return _tensor_digest(model.named_buffers())


def is_reference_checkpoint(path) -> bool:
    try:
        return json.loads((Path(path) / "manifest.json").read_text()).get("format") == FORMAT
    except (OSError, ValueError):
        return False


def read_reference_manifest(path) -> dict:
    manifest = json.loads((Path(path) / "manifest.json").read_text())
    if manifest.get("format") != FORMAT:
        raise ValueError(f"not a {FORMAT} checkpoint")
    return manifest


def _held_model_state(model, dp) -> dict:
    """The model entries this rank holds: everything replicated, plus its own sharded parameters."""
    if dp is not None and getattr(dp, "shard_params", False):
        return {**dp.replicated_state(), **dp.owned_sharded_state()}
    return model.state_dict()


def _owned_parameters(optimizer) -> list:
    return [p for part in _parts(optimizer) for g in part.param_groups for p in g["params"]]


# ====================================================================================== saving
def _zero_state(part, p) -> dict:
    """The state a never-stepped parameter would have (the reference allocates it before saving)."""
    if isinstance(part, torch.optim.AdamW):
        return {"step": torch.zeros((), dtype=torch.float32), "exp_avg": torch.zeros_like(p),
                "exp_avg_sq": torch.zeros_like(p)}
    return {"momentum_buffer": torch.zeros_like(p)}


def _group_records(optimizer, logical, names) -> list[dict]:
    """Every group with its hyper-parameters (from the live optimizer) and all of its parameter
    names (from the logical optimizer, which spans every rank's parameters)."""
    records = []
    for live, full in zip([g for part in _parts(optimizer) for g in part.param_groups],
                          [g for part in _parts(logical) for g in part.param_groups]):
        record = {k: to_plain(v.item() if isinstance(v, torch.Tensor) and v.numel() == 1 else v)
                  for k, v in live.items() if k != "params"}
        for key, default in _IMPLEMENTATION_KEYS.items():
            if key in record:
                record[key] = default
        record["params"] = [names[id(p)] for p in full["params"]]
        records.append(record)
    return records


def save_reference_checkpoint(path, model, optimizer, sampler, dp, *, logical, config, progress, manifest_hash,
                              parent=None) -> dict:
    """Collectively write ``path`` in the reference's ``tnlm-dcp-v1`` format; returns its manifest."""
    import torch.distributed.checkpoint as dcp
    rank, world = _group()
    path = Path(path).resolve()
    device_type = next(iter(_held_model_state(model, dp).values())).device.type
    names = _fqns(model)

    def preflight():
        if path.exists():
            raise FileExistsError(f"checkpoint already exists: {path}")
        held = _held_model_state(model, dp)
        assert_finite(held, "model")
        assert_finite(optimizer.state_dict(), "optimizer")
        for module in model.modules():
            for buf in ("acc_count", "acc_sum"):
                value = getattr(module, buf, None)
                if value is not None and bool(torch.as_tensor(value).ne(0).any()):
                    raise ValueError("checkpoint requires committed lagged statistics at a step boundary")
        groups = _group_records(optimizer, logical, names)
        return {"config": to_plain(config), "progress": to_plain(progress), "manifest_hash": manifest_hash,
                "parent": to_plain(parent), "world_size": world, "torch_version": str(torch.__version__),
                "backend": str(dist.get_backend()), "layout": _reference_layout(model, logical, world, device_type),
                "runtime": _runtime_flags(),
                "optimizer_hyperparameters_scope": "informational save-time snapshot; checksummed DCP optimizer "
                                                   "state is recovery authority",
                "optimizer_hyperparameters": _nested_groups(optimizer, groups)}
    shared = _agree("reference checkpoint metadata", _phase("reference checkpoint preflight", preflight))
    buffers = _agree("replicated buffers", _phase("buffer digest", lambda: _buffer_digest(model)))
    local = {"rank": rank, "world_size": world, "rng": rng_capture(), "sampler": sampler.state_dict()}
    _agree("global sampler stream", {"sampler_type": type(sampler).__name__, "stream": local["sampler"].get("stream")})

    def collect():
        state = {f"model.{k}": v.detach() for k, v in _held_model_state(model, dp).items()}
        for part in _parts(optimizer):
            for g in part.param_groups:
                for p in g["params"]:
                    stats = part.state.get(p) or _zero_state(part, p)
                    for stat, value in stats.items():
                        state[f"optimizer.state.{names[id(p)]}.{stat}"] = value.detach()
        for i, record in enumerate(_group_records(optimizer, logical, names)):
            for key, value in record.items():
                state[f"optimizer.param_groups.{i}.{key}"] = value
        return state
    state = _phase("state collection", collect)

    def staging():
        if rank:
            return None
        estimate = checkpoint_space_estimate({"state": state, "local": local}) * world
        require_checkpoint_space(path.parent, estimate)
        path.parent.mkdir(parents=True, exist_ok=True)
        return tempfile.mkdtemp(prefix=f".{path.name}.tmp-", dir=path.parent)
    box = [_phase("staging directory", staging)]
    dist.broadcast_object_list(box, src=0)
    stage = Path(box[0])
    try:
        _phase("DCP save", lambda: dcp.save(state, checkpoint_id=stage / "dcp"))

        def write_rank():
            with (stage / f"rank-{rank:05d}.pt").open("wb") as fh:
                torch.save(local, fh)
                fh.flush()
                os.fsync(fh.fileno())
        _phase("rank recovery save", write_rank)
        dist.barrier()

        def publish():
            if rank:
                return None
            files = {}
            for item in sorted(stage.rglob("*")):
                if item.is_file():
                    with item.open("rb") as fh:
                        os.fsync(fh.fileno())
                    files[str(item.relative_to(stage))] = {"sha256": file_sha256(item), "bytes": item.stat().st_size}
            manifest = {"format": FORMAT, **shared, "files": files, "code": code_identity(),
                        "disk_admission": None, "replicated_buffers_sha256": buffers,
                        "created_utc": datetime.now(timezone.utc).isoformat(), "replay_scope": _REPLAY_SCOPE}
            with (stage / "manifest.json").open("w") as fh:
                json.dump(manifest, fh, sort_keys=True, indent=2, allow_nan=False)
                fh.write("\n")
                fh.flush()
                os.fsync(fh.fileno())
            for d in sorted((p for p in stage.rglob("*") if p.is_dir()), reverse=True):
                fsync_dir(d)
            fsync_dir(stage)
            publish_dir(stage, path)
            return manifest
        box = [_phase("atomic publication", publish)]
        dist.broadcast_object_list(box, src=0)
        return box[0]
    finally:
        if rank == 0 and stage.exists():
            shutil.rmtree(stage, ignore_errors=True)


def _nested_groups(optimizer, records) -> list:
    """The manifest's informational per-child hyper-parameter lists (``params`` omitted)."""
    out, i = [], 0
    for part in _parts(optimizer):
        n = len(part.param_groups)
        out.append([{k: v for k, v in r.items() if k != "params"} for r in records[i:i + n]])
        i += n
    return out


# ====================================================================================== loading
def _verify_files(path: Path, manifest: dict, world: int):
    files = manifest["files"]
    required = {f"rank-{i:05d}.pt" for i in range(world)} | {"dcp/.metadata"}
    if not required <= set(files) or not any(name.endswith(".distcp") for name in files):
        raise ValueError("incomplete checkpoint shard set")
    present = {str(p.relative_to(path)) for p in path.rglob("*") if p.is_file()} - {"manifest.json"}
    if present != set(files):
        raise ValueError("checkpoint file set differs from manifest")
    for name, entry in files.items():
        rel = Path(name)
        if rel.is_absolute() or ".." in rel.parts:
            raise ValueError("invalid checkpoint artifact path")
        if (path / rel).stat().st_size != entry["bytes"] or file_sha256(path / rel) != entry["sha256"]:
            raise ValueError(f"checkpoint checksum mismatch: {name}")


def _comparable(layout: dict) -> dict:
    """What must agree between a saved layout and this job's (shapes, dtypes and groups; the
    sharding placement does not matter to a resharding load)."""
    return {"model": {k: (v["shape"], v["dtype"]) for k, v in layout["model"].items()},
            "optimizer": layout["optimizer"], "parameter_groups": layout["parameter_groups"],
            "children": [c["parameter_groups"] for c in layout.get("optimizer_children", [])]}


def _check_hyperparameters(optimizer, loaded_groups: list[dict]):
    live = [g for part in _parts(optimizer) for g in part.param_groups]
    if len(live) != len(loaded_groups):
        raise ValueError("checkpoint optimizer group count differs")
    for i, (mine, theirs) in enumerate(zip(live, loaded_groups)):
        for key in _MATH_KEYS:
            if key in mine and key in theirs and to_plain(mine[key]) != to_plain(theirs[key]):
                raise ValueError(f"checkpoint optimizer group {i} differs in {key}")


def load_reference_checkpoint(path, model, optimizer, sampler, dp, *, logical, expected_manifest_hash=None,
                              config_validator=None, restore_rng=True) -> dict:
    """Collectively restore a ``tnlm-dcp-v1`` checkpoint of the same world size: model, this rank's
    optimizer state, sampler cursor and RNG.  Nothing live changes until every check has passed."""
    import torch.distributed.checkpoint as dcp
    rank, world = _group()
    path = Path(path).resolve()
    device_type = next(iter(_held_model_state(model, dp).values())).device.type

    def verify():
        manifest = read_reference_manifest(path)
        if manifest["world_size"] != world:
            raise ValueError(f"checkpoint world size {manifest['world_size']} != {world}")
        if manifest["torch_version"] != str(torch.__version__):
            raise ValueError("checkpoint torch version differs")
        if _comparable(manifest["layout"]) != _comparable(_reference_layout(model, logical, world, device_type)):
            raise ValueError("checkpoint model/optimizer layout differs")
        if expected_manifest_hash is not None and manifest["manifest_hash"] != expected_manifest_hash:
            raise ValueError("data manifest hash mismatch")
        if rank == 0:
            _verify_files(path, manifest, world)
        compat = config_validator(manifest["config"]) if config_validator is not None else None
        return manifest, compat
    manifest, compat = _phase("reference checkpoint verification", verify)
    _agree("reference checkpoint identity", manifest["replicated_buffers_sha256"])

    def rank_state():
        local = torch.load(path / f"rank-{rank:05d}.pt", map_location="cpu", weights_only=False)
        if local["rank"] != rank or local["world_size"] != world:
            raise ValueError("rank recovery identity mismatch")
        if restore_rng:
            rng_check(local["rng"])
        copy.copy(sampler).load_state_dict(local["sampler"])  # a cursor this sampler accepts
        return local
    local = _phase("rank recovery verification", rank_state)
    _agree("restored global sampler stream", {"sampler_type": type(sampler).__name__,
                                             "stream": local["sampler"].get("stream")})
    names = _fqns(model)

    def request():
        meta = dcp.FileSystemReader(str(path / "dcp")).read_metadata().state_dict_metadata
        wanted = {f"model.{k}": torch.empty(v.shape, dtype=v.dtype) for k, v in _held_model_state(model, dp).items()}
        for p in _owned_parameters(optimizer):
            prefix = f"optimizer.state.{names[id(p)]}."
            for key, entry in meta.items():
                if key.startswith(prefix) and "." not in key[len(prefix):]:
                    wanted[key] = torch.empty(tuple(entry.size), dtype=entry.properties.dtype)
        for key in meta:
            if key.startswith("optimizer.param_groups."):
                wanted[key] = None
        return wanted
    state = _phase("load request", request)
    _phase("DCP load", lambda: dcp.load(state, checkpoint_id=path / "dcp"))

    def stage():
        assert_finite({k: v for k, v in state.items() if isinstance(v, torch.Tensor)}, "checkpoint")
        groups: dict[int, dict] = {}
        for key, value in state.items():
            if key.startswith("optimizer.param_groups."):
                index, field = key[len("optimizer.param_groups."):].split(".", 1)
                groups.setdefault(int(index), {})[field] = value
        loaded = [groups[i] for i in sorted(groups)]
        _check_hyperparameters(optimizer, loaded)
        by_name = [set(g["params"]) for g in loaded]
        live = [g for part in _parts(optimizer) for g in part.param_groups]
        if any(names[id(p)] not in by_name[i] for i, g in enumerate(live) for p in g["params"]):
            raise ValueError("a parameter sits in another optimizer group in the checkpoint")
        return loaded
    _phase("loaded state validation", stage)

    def install():
        with torch.no_grad():
            held = _held_model_state(model, dp)
            for k, v in held.items():
                v.copy_(state[f"model.{k}"])
        for part in _parts(optimizer):
            restored, index = {"state": {}, "param_groups": []}, 0
            for g in part.param_groups:
                ids = []
                for p in g["params"]:
                    prefix = f"optimizer.state.{names[id(p)]}."
                    stats = {k[len(prefix):]: v for k, v in state.items() if k.startswith(prefix)}
                    if stats:
                        restored["state"][index] = stats
                    ids.append(index)
                    index += 1
                restored["param_groups"].append({**{k: v for k, v in g.items() if k != "params"}, "params": ids})
            part.load_state_dict(restored)
        sampler.load_state_dict(local["sampler"])
        if restore_rng:
            rng_restore(local["rng"])
    _phase("state installation", install)
    if dp is not None and getattr(dp, "shard_params", False):
        dp.gather_params()
    restored = _buffer_digest(model)
    _agree("restored replicated buffers", restored)
    if restored != manifest["replicated_buffers_sha256"]:
        raise ValueError("restored buffers differ from the checkpoint")
    out = {**manifest, **{k: local[k] for k in ("rank", "sampler")}}
    if compat is not None:
        out["config_compatibility"] = compat
    return out
