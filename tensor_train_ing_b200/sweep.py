"""Sequential, fail-closed execution of a frozen candidate sweep (reference tnlm/sweep.py:98-459).

For every candidate, in order: a fresh full-rung parent run; optionally a cooldown fork from the
parent's 90% milestone (first optimizer boundary at or above 90% of the rung) to the rung's exact
token endpoint; a held-out evaluation of the selected endpoint.  Then paired comparisons of every
candidate against the reference candidate and a training summary.

``sweep.json`` is the journal: the frozen identity (configs, data manifests, controls, source
hashes) and the status, artifact hashes, result and billing of each stage.  A re-invocation reuses
a completed stage only after re-hashing every artifact; a failed or interrupted stage is never
retried automatically.  With ``prune_completed_intermediates`` the milestone / recovery payloads of
a fully evaluated candidate are deleted after a durable plan is journaled (manifests are kept).
"""
from __future__ import annotations

import copy
import fcntl
import hashlib
import json
import math
import os
from pathlib import Path

import torch

from .checkpoint_plan import checkpoint_storage_plan
from .checkpoint_storage import require_checkpoint_space
from .config import Config, ModelConfig, TrainConfig
from .evaluate import compare_evaluations, evaluate_checkpoint
from .reporting import summarize_runs
from .search import plan_sweep
from .sweep_retention import intermediate_payload, reject_symlink_chain, retention_forecast, unlink_payload
from .train import train_run

_RESERVED = ("summary", "sweep.json", "sweep.json.tmp", "comparisons")


def _sha(path) -> str:
    h = hashlib.sha256()
    with Path(path).open("rb") as fh:
        for block in iter(lambda: fh.read(8 << 20), b""):
            h.update(block)
    return h.hexdigest()


def _sources() -> dict:
    pkg = Path(__file__).parent
    return {str(p.relative_to(pkg)): _sha(p) for p in sorted(pkg.rglob("*.py"))}


def _cfg(value) -> Config:
    value = copy.deepcopy(value)
    return Config(model=ModelConfig(**value["model"]), train=TrainConfig(**value["train"]), raw=value)


def _snapshot(path) -> dict:
    files = {}
    for item in sorted(Path(path).rglob("*")):
        if item.is_symlink():
            raise ValueError("stage artifacts must not be symlinks")
        if item.is_file():
            files[str(item.relative_to(path))] = {"bytes": item.stat().st_size, "sha256": _sha(item)}
    if not files:
        raise ValueError("stage did not publish artifacts")
    return files


def _atomic(path, value):
    tmp = path.with_name(path.name + ".tmp")
    with tmp.open("w") as fh:
        json.dump(value, fh, sort_keys=True, indent=2, allow_nan=False)
        fh.write("\n")
        fh.flush()
        os.fsync(fh.fileno())
    os.replace(tmp, path)
    fd = os.open(path.parent, os.O_RDONLY)
    try:
        os.fsync(fd)
    finally:
        os.close(fd)


def _checkpoint(path, cfg, expected_tokens, *, manifest_hash, cooldown_steps=None, parent=None) -> dict:
    """Gate a stage's checkpoint: schema, checksum, config, token endpoint, parent and cooldown horizon."""
    path = Path(path)
    manifest = json.loads((path / "manifest.json").read_text())
    if manifest.get("format_version") != 1 or manifest.get("data_manifest_hash") != manifest_hash:
        raise ValueError("checkpoint schema/data identity mismatch")
    info = manifest["files"]["state.pt"]
    if (path / "state.pt").stat().st_size != info["bytes"] or _sha(path / "state.pt") != info["sha256"]:
        raise ValueError("checkpoint checksum mismatch")
    payload = torch.load(path / "state.pt", map_location="cpu", weights_only=False, mmap=True)
    if (payload["config"] != cfg or payload["progress"]["tokens"] != expected_tokens
            or payload.get("manifest_hash") != manifest_hash or payload.get("parent") != parent
            or manifest.get("parent") != parent):
        raise ValueError("stage checkpoint config/token endpoint mismatch")
    progress, extra = payload["progress"], payload.get("extra") or {}
    if cooldown_steps is None:
        if extra.get("cooldown_steps") is not None:
            raise ValueError("parent/branch checkpoint is already cooled")
    elif (extra.get("cooldown_steps") != cooldown_steps or extra.get("cooldown_end_tokens") != expected_tokens
          or progress.get("scheduler_step") != cooldown_steps or progress.get("cooldown_end_tokens") != expected_tokens):
        raise ValueError("cooldown checkpoint horizon/endpoint mismatch")
    return {"path": str(path), "tokens": expected_tokens, "manifest_sha256": _sha(path / "manifest.json"),
            "state_sha256": info["sha256"]}


def _plan(base_cfg, candidates, out, *, max_seconds, evaluation_max_seconds, device, cooldown, max_prediction_tokens,
          bootstrap_samples, reference_candidate, prune, canary):
    context = base_cfg.raw.get("data", {}).get("context", 512)
    if type(context) is not int or context <= 0:
        raise ValueError("evaluation context must be positive integer")
    frozen = plan_sweep(base_cfg, candidates)
    if any(r["name"] in _RESERVED for r in frozen["runs"]):
        raise ValueError("candidate name is reserved for sweep orchestration")
    reference_candidate = frozen["runs"][0]["name"] if reference_candidate is None else reference_candidate
    if reference_candidate not in {r["name"] for r in frozen["runs"]}:
        raise ValueError("reference_candidate must name a declared candidate")
    flags = [r["config"].get("project", {}).get("dry_run", True) for r in frozen["runs"]]
    if any(type(f) is not bool for f in flags) or len(set(flags)) != 1:
        raise ValueError("all candidates must share an explicit Boolean dry_run policy")
    dry = flags[0]
    trajectories, val_hashes, eval_seeds, storage = [], set(), set(), 0
    for run in frozen["runs"]:
        cfg = _cfg(run["config"])
        data = cfg.raw.get("data", {})
        if cooldown and cfg.train.schedule != "constant_with_separate_cooldown":
            raise ValueError("separate sweep cooldown requires constant_with_separate_cooldown; use --no-cooldown for cosine")
        identities = {}
        for label, value in (("training", data.get("manifest")),
                             ("validation", cfg.raw.get("evaluation", {}).get("validation_manifest", data.get("manifest")))):
            p = Path(value).resolve() if value is not None else None
            if p is not None and p.is_dir():
                p /= "manifest.json"
            if p is None or not p.is_file():
                if not dry:
                    raise ValueError(f"{label} manifest must exist before execution")
                identities[label] = {"path": str(p) if p else None, "sha256": None}
            else:
                identities[label] = {"path": str(p), "sha256": _sha(p)}
        val_hashes.add(identities["validation"]["sha256"])
        seed = cfg.raw.get("evaluation", {}).get("seed", 0)
        if type(seed) is not int or seed < 0:
            raise ValueError("evaluation seed must be a nonnegative integer")
        eval_seeds.add(seed)
        limit, batch = cfg.train.rung_total_tokens, cfg.train.global_prediction_tokens_per_update
        if canary and (limit + batch - 1) // batch < canary["warmup_steps"] + canary["measured_steps"]:
            raise ValueError("parent horizon cannot complete the requested throughput canary")
        threshold = 9 * limit // 10
        branch = ((threshold + batch - 1) // batch) * batch
        if cooldown and not 0 < branch < limit:
            raise ValueError("rung has no proper optimizer-boundary 90% cooldown branch")
        horizon = (limit - branch + batch - 1) // batch if cooldown else None
        parent_plan = checkpoint_storage_plan(cfg)
        cooled_plan = (checkpoint_storage_plan(cfg, start_tokens=branch, token_limit=limit, max_steps=horizon,
                                               cooldown=True) if cooldown else None)
        storage += parent_plan["required_additional_bytes"] + (cooled_plan["required_additional_bytes"] if cooled_plan else 0)
        rate = cfg.raw.get("project", {}).get("gpu_hourly_rate_usd")
        margin = cfg.raw.get("project", {}).get("cost_margin_fraction", .1)
        if isinstance(margin, bool) or not isinstance(margin, (int, float)) or not math.isfinite(margin) or margin < 0:
            raise ValueError("cost margin must be finite nonnegative")
        cap = float(rate) * ((2 if cooldown else 1) * max_seconds + evaluation_max_seconds) / 3600 if rate is not None else None
        trajectories.append({
            "name": run["name"], "config": run["config"], "config_sha256": run["config_sha256"], "data": identities,
            "paths": {"parent": str(out / run["name"] / "parent"),
                      "cooldown": str(out / run["name"] / "cooldown") if cooldown else None,
                      "evaluation": str(out / run["name"] / "evaluation")},
            "runtime_cap_based_usd": cap, "reservation_cap_based_usd": cap * (1 + margin) if cap is not None else None,
            "tokens": limit, "parent_steps": (limit + batch - 1) // batch, "branch_threshold": threshold,
            "branch_tokens": branch if cooldown else None, "cooldown_steps": horizon,
            "cooldown_end_tokens": limit if cooldown else None, "parent_storage_plan": parent_plan,
            "cooldown_storage_plan": cooled_plan})
    if len(eval_seeds) != 1:
        raise ValueError("sweep candidates require one identical evaluation seed")
    if len(val_hashes) != 1:
        raise ValueError("sweep candidates require one identical frozen validation manifest")
    seed = next(iter(eval_seeds))
    identity = {"version": 1, "out_dir": str(out), "trajectories": trajectories,
                "controls": {"throughput_canary": canary, "max_seconds": max_seconds,
                             "evaluation_max_seconds": evaluation_max_seconds, "device": device, "cooldown": cooldown,
                             "max_prediction_tokens": max_prediction_tokens, "bootstrap_samples": bootstrap_samples,
                             "evaluation_context": context, "evaluation_seed": seed, "comparison_seed": seed,
                             "reference_candidate": reference_candidate, "prune_completed_intermediates": prune},
                "runtime_source_sha256": _sources()}
    digest = hashlib.sha256(json.dumps(identity, sort_keys=True, separators=(",", ":"), allow_nan=False).encode()).hexdigest()
    forecast = retention_forecast(trajectories) if prune else None
    if forecast is not None:
        storage = forecast["required_additional_bytes"]
    total = lambda key: (sum(r[key] for r in trajectories)  # noqa: E731
                         if all(r[key] is not None for r in trajectories) else None)
    return {"kind": "frozen_sweep_execution", "dry_run": dry, "identity": identity, "identity_sha256": digest,
            "required_additional_bytes": storage, "retention_forecast": forecast,
            "retention_scope": ("final, initial and all metadata retained; completed milestone/recovery payloads "
                                "deleted after evaluation" if prune else "all completed stage artifacts retained"),
            "comparison_pairs": [{"reference": reference_candidate, "candidate": r["name"]}
                                 for r in trajectories if r["name"] != reference_candidate],
            "runtime_cap_based_usd": total("runtime_cap_based_usd"),
            "reservation_cap_based_usd": total("reservation_cap_based_usd"),
            "scope": "full configured schedule plus optional cooldown and evaluation stages; no final test",
            "cost_scope": "cap-based estimates; each stage admits and bills its actual elapsed time"}


def run_sweep(base_cfg, candidates, out_dir, *, max_seconds, evaluation_max_seconds, device="cuda", cooldown=True,
              max_prediction_tokens=1_000_000, bootstrap_samples=1000, reference_candidate=None,
              prune_completed_intermediates=False, canary_steps=0, min_tokens_per_second=None, canary_warmup_steps=12):
    from .throughput_canary import ThroughputCanary
    if type(canary_steps) is not int or canary_steps < 0:
        raise ValueError("canary_steps must be a nonnegative integer")
    canary = None
    if canary_steps:
        ThroughputCanary(canary_steps, min_tokens_per_second, canary_warmup_steps)  # validates the controls
        canary = {"measured_steps": canary_steps, "min_tokens_per_second": min_tokens_per_second,
                  "warmup_steps": canary_warmup_steps,
                  "scope": "first measured parent updates after the excluded warm-up; no extra trajectory"}
    elif min_tokens_per_second is not None or canary_warmup_steps != 12:
        raise ValueError("canary threshold/warmup requires positive canary_steps")
    if type(prune_completed_intermediates) is not bool:
        raise ValueError("prune_completed_intermediates must be Boolean")
    for v in (max_seconds, evaluation_max_seconds):
        if isinstance(v, bool) or not isinstance(v, (int, float)) or not math.isfinite(v) or v <= 0:
            raise ValueError("stage time caps must be finite positive numbers")
    if type(cooldown) is not bool or type(max_prediction_tokens) is not int or max_prediction_tokens <= 0:
        raise ValueError("cooldown must be bool and prediction budget positive integer")
    if type(bootstrap_samples) is not int or not 0 <= bootstrap_samples <= 100_000:
        raise ValueError("bootstrap_samples must be in [0,100000]")
    out = Path(out_dir).resolve()
    planned = _plan(base_cfg, candidates, out, max_seconds=max_seconds, evaluation_max_seconds=evaluation_max_seconds,
                    device=str(torch.device(device)), cooldown=cooldown, max_prediction_tokens=max_prediction_tokens,
                    bootstrap_samples=bootstrap_samples, reference_candidate=reference_candidate,
                    prune=prune_completed_intermediates, canary=canary)
    if planned["dry_run"]:
        return planned
    identity, digest = planned["identity"], planned["identity_sha256"]
    trajectories = identity["trajectories"]
    controls = identity["controls"]
    out.mkdir(parents=True, exist_ok=True)
    with (out / ".sweep.lock").open("a") as lock:
        try:
            fcntl.flock(lock, fcntl.LOCK_EX | fcntl.LOCK_NB)
        except BlockingIOError as exc:
            raise RuntimeError("another sweep invocation holds the output lock") from exc
        jpath = out / "sweep.json"
        if jpath.exists():
            journal = json.loads(jpath.read_text())
            if journal.get("identity_sha256") != digest or journal.get("identity") != identity:
                raise ValueError("frozen sweep identity mismatch")
            if any(s["status"] != "complete" for s in journal["stages"].values()):
                raise RuntimeError("interrupted/failed sweep stage requires explicit recovery; automatic retry forbidden")
        else:
            if any(p.name != ".sweep.lock" for p in out.iterdir()):
                raise FileExistsError("sweep output contains unjournaled artifacts")
            journal = {**planned, "stages": {}, "prune_operations": {}, "status": "pending"}
            _atomic(jpath, journal)

        def bill(ledger, directory):
            row = json.loads(Path(ledger).read_text())["runs"][str(Path(directory).resolve())]
            if row.get("status") != "complete" or row.get("reserved_usd") != 0:
                raise ValueError("stage billing is not terminal complete")
            return {"ledger": str(ledger), "run_id": str(Path(directory).resolve()), "spent_usd": row["spent_usd"]}

        def check_inputs(run):
            if _sources() != identity["runtime_source_sha256"]:
                raise ValueError("frozen runtime sources changed during sweep")
            for item in run["data"].values():
                if _sha(item["path"]) != item["sha256"]:
                    raise ValueError("frozen data manifest changed before stage")

        def prune_files(run):
            files = {}
            for phase in ("parent", "cooldown"):
                key = f"{run['name']}/{phase}"
                for rel, info in journal["stages"].get(key, {}).get("artifacts", {}).items():
                    if intermediate_payload(rel):
                        files[f"{key}/{rel}"] = {"stage": key, "artifact": rel, **info}
            return files

        def verify_stage(key, directory, ledger=None):
            record = journal["stages"][key]
            reject_symlink_chain(out, directory)
            actual = _snapshot(directory)
            expected = dict(record["artifacts"])
            for op in journal.get("prune_operations", {}).values():
                for item in op["files"].values():
                    if item["stage"] == key and item["artifact"] not in actual:
                        expected.pop(item["artifact"], None)
                    elif item["stage"] == key and op["status"] == "complete":
                        raise ValueError("completed prune payload unexpectedly reappeared")
            if actual != expected:
                raise ValueError(f"completed stage artifact hash mismatch: {key}")
            if json.loads((Path(directory) / ".sweep-stage.json").read_text()) != record["result"]:
                raise ValueError("cached stage result differs from frozen artifact")
            if ledger is not None and bill(ledger, directory) != record["billing"]:
                raise ValueError("completed stage billing identity changed")
            return record["result"]

        def stage(key, directory, callback, ledger=None):
            directory = Path(directory)
            if key in journal["stages"]:
                return verify_stage(key, directory, ledger)
            if directory.exists():
                raise FileExistsError(f"unjournaled stage output: {directory}")
            journal["stages"][key] = {"status": "running"}
            journal["status"] = "running"
            _atomic(jpath, journal)
            try:
                result = callback()
                if _sources() != identity["runtime_source_sha256"]:
                    raise ValueError("frozen runtime sources changed during sweep")
                billing = bill(ledger, directory) if ledger is not None else None
                _atomic(directory / ".sweep-stage.json", result)
                journal["stages"][key] = {"status": "complete", "artifacts": _snapshot(directory), "result": result,
                                          "billing": billing}
                _atomic(jpath, journal)
                return result
            except BaseException as exc:
                journal["stages"][key] = {"status": "failed", "error": f"{type(exc).__name__}: {exc}"}
                journal["status"] = "failed"
                _atomic(jpath, journal)
                raise

        def prune(run):
            ledger = Path(run["config"]["project"]["spend_ledger"])
            with Path(str(ledger) + ".lock").open("a") as llock:  # the ledger's own admission lock
                fcntl.flock(llock, fcntl.LOCK_EX)
                keys = [f"{run['name']}/parent", f"{run['name']}/evaluation"]
                if run["cooldown_storage_plan"] is not None:
                    keys.append(f"{run['name']}/cooldown")
                for key in keys:
                    verify_stage(key, out / key, ledger)
                slated = {str((out / rel).parent) for rel in prune_files(run)}
                own = {str(out / k) for k in keys}
                for run_id, row in json.loads(ledger.read_text())["runs"].items():
                    ref = row.get("parent_checkpoint")
                    if (run_id not in own and ref is not None and str(Path(ref).resolve()) in slated
                            and (row.get("status") != "complete" or row.get("reserved_usd") != 0)):
                        raise ValueError("an active run pins a slated checkpoint payload")
                ops = journal.setdefault("prune_operations", {})
                if run["name"] not in ops:
                    files = prune_files(run)
                    ops[run["name"]] = {"status": "planned", "files": files,
                                        "original_payload_bytes": sum(i["bytes"] for i in files.values())}
                    _atomic(jpath, journal)  # durable authorisation before any unlink
                op = ops[run["name"]]
                if op["status"] != "complete":
                    for rel, item in op["files"].items():
                        unlink_payload(out, rel, item)
                    op["status"] = "complete"
                    _atomic(jpath, journal)

        for run in trajectories:
            if journal.get("prune_operations", {}).get(run["name"], {}).get("status") == "planned":
                prune(run)
        if journal["status"] != "complete":
            pending = sum(r["parent_storage_plan"]["required_additional_bytes"] * (f"{r['name']}/parent" not in journal["stages"])
                          + (r["cooldown_storage_plan"]["required_additional_bytes"]
                             if r["cooldown_storage_plan"] and f"{r['name']}/cooldown" not in journal["stages"] else 0)
                          for r in trajectories)
            if prune_completed_intermediates:
                fc = retention_forecast(trajectories, journal["stages"])
                pending = fc["required_additional_bytes"]
                journal["pending_retention_forecast"] = fc
            journal["disk_admission"] = require_checkpoint_space(out, pending)
            _atomic(jpath, journal)
        training_dirs, reports = [], []
        for run in trajectories:
            name, cfg = run["name"], _cfg(run["config"])
            ledger = cfg.raw["project"]["spend_ledger"]
            parent_dir = out / name / "parent"

            def parent(run=run, cfg=cfg, parent_dir=parent_dir):
                check_inputs(run)
                observer = (ThroughputCanary(canary["measured_steps"], canary["min_tokens_per_second"],
                                             canary["warmup_steps"]) if canary else None)
                result = train_run(cfg, parent_dir, max_steps=run["parent_steps"], max_seconds=max_seconds,
                                   device=controls["device"], **({"_throughput_canary": observer} if observer else {}))
                if Path(result["checkpoint"]).resolve() != (parent_dir / "final").resolve():
                    raise ValueError("parent returned checkpoint outside expected final directory")
                mh = run["data"]["training"]["sha256"]
                final = _checkpoint(result["checkpoint"], run["config"], run["tokens"], manifest_hash=mh)
                branch = (_checkpoint(parent_dir / f"milestone-{run['branch_threshold']:012d}", run["config"],
                                      run["branch_tokens"], manifest_hash=mh) if cooldown else None)
                return {"checkpoint": final, "branch": branch,
                        **({"throughput_canary": observer.report()} if observer else {})}
            pres = stage(f"{name}/parent", parent_dir, parent, ledger)
            training_dirs.append(parent_dir)
            selected = pres["checkpoint"]
            if cooldown:
                cooled_dir = out / name / "cooldown"

                def cooled(run=run, cfg=cfg, cooled_dir=cooled_dir, pres=pres):
                    check_inputs(run)
                    result = train_run(cfg, cooled_dir, max_steps=run["cooldown_steps"], max_seconds=max_seconds,
                                       device=controls["device"], resume=pres["branch"]["path"],
                                       cooldown_steps=run["cooldown_steps"], cooldown_end_tokens=run["tokens"])
                    if Path(result["checkpoint"]).resolve() != (cooled_dir / "final").resolve():
                        raise ValueError("cooldown returned checkpoint outside expected final directory")
                    return _checkpoint(result["checkpoint"], run["config"], run["tokens"],
                                       cooldown_steps=run["cooldown_steps"], manifest_hash=run["data"]["training"]["sha256"],
                                       parent={"path": pres["branch"]["path"],
                                               "manifest_sha256": pres["branch"]["manifest_sha256"]})
                selected = stage(f"{name}/cooldown", cooled_dir, cooled, ledger)
                training_dirs.append(cooled_dir)
            eval_dir = out / name / "evaluation"

            def evaluate(run=run, cfg=cfg, eval_dir=eval_dir, selected=selected):
                check_inputs(run)
                rep = evaluate_checkpoint(cfg, selected["path"], eval_dir, context=controls["evaluation_context"],
                                          max_prediction_tokens=max_prediction_tokens,
                                          max_seconds=evaluation_max_seconds, device=controls["device"],
                                          bootstrap_samples=bootstrap_samples)
                if (rep.get("kind") != "held_out_validation" or not rep["frozen_state"]["unchanged"]
                        or rep["validation_manifest_sha256"] != run["data"]["validation"]["sha256"]
                        or rep["checkpoint_manifest_sha256"] != selected["manifest_sha256"]
                        or rep["checkpoint_state_sha256"] != selected["state_sha256"]):
                    raise ValueError("evaluation protocol/state mismatch")
                return {k: rep[k] for k in ("checkpoint_manifest_sha256", "checkpoint_state_sha256",
                                            "validation_manifest_sha256", "target_plan_sha256",
                                            "available_prefix_plan_sha256", "prediction_tokens", "ce")}
            reports.append({"name": name, **stage(f"{name}/evaluation", eval_dir, evaluate, ledger)})
            if prune_completed_intermediates:
                prune(run)
        if len({(r["target_plan_sha256"], r["available_prefix_plan_sha256"], r["prediction_tokens"]) for r in reports}) != 1:
            raise ValueError("candidate validation targets/prefixes differ; comparison rejected")
        ref = controls["reference_candidate"]
        comparisons = []
        for run in trajectories:
            if run["name"] == ref:
                continue
            cdir = out / "comparisons" / run["name"]

            def compare(run=run, cdir=cdir):
                rep = compare_evaluations(out / ref / "evaluation" / "evaluation.json",
                                          out / run["name"] / "evaluation" / "evaluation.json", cdir,
                                          bootstrap_samples=bootstrap_samples, seed=controls["comparison_seed"])
                return {"reference_candidate": ref, "candidate": run["name"], "path": str(cdir / "comparison.json"),
                        "delta_ce_right_minus_left": rep["delta_ce_right_minus_left"],
                        "delta_ce_95_ci": rep["uncertainty"]["delta_ce_95_ci"], "uncertainty": rep["uncertainty"],
                        "training_comparison": rep["training_comparison"]}
            comparisons.append(stage(f"comparison/{run['name']}", cdir, compare))
        sdir = out / "summary"

        def summarize():
            result = summarize_runs(training_dirs, sdir)
            _atomic(sdir / "validation.json", {"evaluations": reports, "reference_candidate": ref,
                                               "comparisons": comparisons, "automatic_ranking_eligible": False,
                                               "scope": "validation only; one seed per candidate; no promotion"})
            return result
        stage("summary", sdir, summarize)
        journal["status"] = "complete"
        _atomic(jpath, journal)
        return journal
