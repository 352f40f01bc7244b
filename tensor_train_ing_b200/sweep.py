"""Sequential, fail-closed execution of a frozen candidate sweep.  Same stages, journal format and
guarantees as the reference's sweep (tnlm/sweep.py:98-459).

For every candidate, in order: a fresh full-rung parent run; optionally a cooldown fork from the
parent's 90 % milestone (the first optimizer boundary at or above 90 % of the rung) to the rung's
exact token endpoint; a held-out evaluation of the selected endpoint.  Then paired comparisons of
every candidate against the reference candidate and a training summary.

``sweep.json`` is the journal: the frozen identity (configs, data manifests, controls, source
hashes) and, per stage, its status, artifact hashes, result and billing.  A re-invocation reuses a
completed stage only after re-hashing every artifact; a failed or interrupted stage is never
retried automatically.  With ``prune_completed_intermediates`` the milestone / recovery payloads of
a fully evaluated candidate are deleted after a durable plan is journaled (manifests are kept).

The pieces: ``_plan`` freezes the identity (one ``_trajectory`` per candidate); ``_Journal`` owns
``sweep.json`` and runs or re-verifies one stage at a time; ``_Sweep`` holds the stage bodies.
"""
from __future__ import annotations

import copy
import fcntl
import json
import math
from pathlib import Path
from typing import Callable

import torch

from .checkpoint_plan import checkpoint_storage_plan
from .checkpoint_storage import require_checkpoint_space
from .config import Config, ModelConfig, TrainConfig
from .durable import write_json
from .evaluate import compare_evaluations, evaluate_checkpoint
from .hashing import canonical_sha256, file_sha256
from .reporting import summarize_runs
from .search import plan_sweep
from .sweep_retention import intermediate_payload, reject_symlink_chain, retention_forecast, unlink_payload
from .train import train_run

_RESERVED = ("summary", "sweep.json", "sweep.json.tmp", "comparisons")
_STAGE_RESULT = ".sweep-stage.json"


def _sources() -> dict:
    pkg = Path(__file__).parent
    return {str(p.relative_to(pkg)): file_sha256(p) for p in sorted(pkg.rglob("*.py"))}


def _config(recorded: dict) -> Config:
    recorded = copy.deepcopy(recorded)
    return Config(model=ModelConfig(**recorded["model"]), train=TrainConfig(**recorded["train"]), raw=recorded)


def _artifacts(directory) -> dict:
    """relative path -> size and sha256 of every file a stage published (symbolic links refused)."""
    files = {}
    for item in sorted(Path(directory).rglob("*")):
        if item.is_symlink():
            raise ValueError("stage artifacts must not be symlinks")
        if item.is_file():
            files[str(item.relative_to(directory))] = {"bytes": item.stat().st_size, "sha256": file_sha256(item)}
    if not files:
        raise ValueError("stage did not publish artifacts")
    return files


def _gate_checkpoint(path, recorded_cfg, tokens, *, manifest_hash, cooldown_steps=None, parent=None) -> dict:
    """A stage's checkpoint must match its manifest, the frozen config, the token endpoint, the
    parent and (for a cooldown) the cooldown horizon; returns its identity for the journal."""
    path = Path(path)
    manifest = json.loads((path / "manifest.json").read_text())
    if manifest.get("format_version") != 1 or manifest.get("data_manifest_hash") != manifest_hash:
        raise ValueError("checkpoint schema/data identity mismatch")
    state_entry = manifest["files"]["state.pt"]
    if (path / "state.pt").stat().st_size != state_entry["bytes"] or file_sha256(path / "state.pt") != state_entry["sha256"]:
        raise ValueError("checkpoint checksum mismatch")
    payload = torch.load(path / "state.pt", map_location="cpu", weights_only=False, mmap=True)
    progress, extra = payload["progress"], payload.get("extra") or {}
    if (payload["config"] != recorded_cfg or progress["tokens"] != tokens or payload.get("manifest_hash") != manifest_hash
            or payload.get("parent") != parent or manifest.get("parent") != parent):
        raise ValueError("stage checkpoint config/token endpoint mismatch")
    if cooldown_steps is None:
        if extra.get("cooldown_steps") is not None:
            raise ValueError("parent/branch checkpoint is already cooled")
    elif (extra.get("cooldown_steps"), extra.get("cooldown_end_tokens"), progress.get("scheduler_step"),
          progress.get("cooldown_end_tokens")) != (cooldown_steps, tokens, cooldown_steps, tokens):
        raise ValueError("cooldown checkpoint horizon/endpoint mismatch")
    return {"path": str(path), "tokens": tokens, "manifest_sha256": file_sha256(path / "manifest.json"),
            "state_sha256": state_entry["sha256"]}


def _terminal_billing(ledger, directory) -> dict:
    run_id = str(Path(directory).resolve())
    row = json.loads(Path(ledger).read_text())["runs"][run_id]
    if row.get("status") != "complete" or row.get("reserved_usd") != 0:
        raise ValueError("stage billing is not terminal complete")
    return {"ledger": str(ledger), "run_id": run_id, "spent_usd": row["spent_usd"]}


# ====================================================================================== planning
def _manifest_identity(label, value, dry) -> dict:
    path = Path(value).resolve() if value is not None else None
    if path is not None and path.is_dir():
        path /= "manifest.json"
    if path is not None and path.is_file():
        return {"path": str(path), "sha256": file_sha256(path)}
    if not dry:
        raise ValueError(f"{label} manifest must exist before execution")
    return {"path": str(path) if path else None, "sha256": None}


def _trajectory(run, out: Path, *, dry, cooldown, canary, max_seconds, evaluation_max_seconds) -> dict:
    """One candidate's frozen trajectory: data identities, stage paths, token endpoints, storage
    plans and cap-based cost."""
    cfg = _config(run["config"])
    data, project = cfg.raw.get("data", {}), cfg.raw.get("project", {})
    if cooldown and cfg.train.schedule != "constant_with_separate_cooldown":
        raise ValueError("separate sweep cooldown requires constant_with_separate_cooldown; use --no-cooldown for cosine")
    identities = {"training": _manifest_identity("training", data.get("manifest"), dry),
                  "validation": _manifest_identity(
                      "validation", cfg.raw.get("evaluation", {}).get("validation_manifest", data.get("manifest")), dry)}
    rung, batch = cfg.train.rung_total_tokens, cfg.train.global_prediction_tokens_per_update
    steps = -(-rung // batch)
    if canary and steps < canary["warmup_steps"] + canary["measured_steps"]:
        raise ValueError("parent horizon cannot complete the requested throughput canary")
    threshold = 9 * rung // 10
    branch = -(-threshold // batch) * batch  # the first optimizer boundary at or above 90 %
    if cooldown and not 0 < branch < rung:
        raise ValueError("rung has no proper optimizer-boundary 90% cooldown branch")
    horizon = -(-(rung - branch) // batch) if cooldown else None
    margin = project.get("cost_margin_fraction", .1)
    if isinstance(margin, bool) or not isinstance(margin, (int, float)) or not math.isfinite(margin) or margin < 0:
        raise ValueError("cost margin must be finite nonnegative")
    rate = project.get("gpu_hourly_rate_usd")
    cap = (float(rate) * ((2 if cooldown else 1) * max_seconds + evaluation_max_seconds) / 3600
           if rate is not None else None)
    home = out / run["name"]
    return {"name": run["name"], "config": run["config"], "config_sha256": run["config_sha256"], "data": identities,
            "paths": {"parent": str(home / "parent"), "cooldown": str(home / "cooldown") if cooldown else None,
                      "evaluation": str(home / "evaluation")},
            "runtime_cap_based_usd": cap, "reservation_cap_based_usd": cap * (1 + margin) if cap is not None else None,
            "tokens": rung, "parent_steps": steps, "branch_threshold": threshold,
            "branch_tokens": branch if cooldown else None, "cooldown_steps": horizon,
            "cooldown_end_tokens": rung if cooldown else None, "parent_storage_plan": checkpoint_storage_plan(cfg),
            "cooldown_storage_plan": (checkpoint_storage_plan(cfg, start_tokens=branch, token_limit=rung,
                                                              max_steps=horizon, cooldown=True) if cooldown else None)}


def _evaluation_seed(run) -> int:
    seed = run["config"].get("evaluation", {}).get("seed", 0)
    if type(seed) is not int or seed < 0:
        raise ValueError("evaluation seed must be a nonnegative integer")
    return seed


def _plan(base_cfg, candidates, out, *, max_seconds, evaluation_max_seconds, device, cooldown, max_prediction_tokens,
          bootstrap_samples, reference_candidate, prune, canary):
    context = base_cfg.raw.get("data", {}).get("context", 512)
    if type(context) is not int or context <= 0:
        raise ValueError("evaluation context must be positive integer")
    frozen = plan_sweep(base_cfg, candidates)
    names = [r["name"] for r in frozen["runs"]]
    if any(n in _RESERVED for n in names):
        raise ValueError("candidate name is reserved for sweep orchestration")
    reference_candidate = names[0] if reference_candidate is None else reference_candidate
    if reference_candidate not in names:
        raise ValueError("reference_candidate must name a declared candidate")
    dry_flags = [r["config"].get("project", {}).get("dry_run", True) for r in frozen["runs"]]
    if any(type(f) is not bool for f in dry_flags) or len(set(dry_flags)) != 1:
        raise ValueError("all candidates must share an explicit Boolean dry_run policy")
    dry = dry_flags[0]
    trajectories = [_trajectory(run, out, dry=dry, cooldown=cooldown, canary=canary, max_seconds=max_seconds,
                                evaluation_max_seconds=evaluation_max_seconds) for run in frozen["runs"]]
    seeds = {_evaluation_seed(run) for run in frozen["runs"]}
    if len(seeds) != 1:
        raise ValueError("sweep candidates require one identical evaluation seed")
    if len({t["data"]["validation"]["sha256"] for t in trajectories}) != 1:
        raise ValueError("sweep candidates require one identical frozen validation manifest")
    seed = seeds.pop()
    identity = {"version": 1, "out_dir": str(out), "trajectories": trajectories,
                "controls": {"throughput_canary": canary, "max_seconds": max_seconds,
                             "evaluation_max_seconds": evaluation_max_seconds, "device": device, "cooldown": cooldown,
                             "max_prediction_tokens": max_prediction_tokens, "bootstrap_samples": bootstrap_samples,
                             "evaluation_context": context, "evaluation_seed": seed, "comparison_seed": seed,
                             "reference_candidate": reference_candidate, "prune_completed_intermediates": prune},
                "runtime_source_sha256": _sources()}
    forecast = retention_forecast(trajectories) if prune else None
    storage = (forecast["required_additional_bytes"] if forecast is not None else
               sum(t["parent_storage_plan"]["required_additional_bytes"]
                   + (t["cooldown_storage_plan"]["required_additional_bytes"] if t["cooldown_storage_plan"] else 0)
                   for t in trajectories))

    def total(key):
        values = [t[key] for t in trajectories]
        return sum(values) if None not in values else None
    return {"kind": "frozen_sweep_execution", "dry_run": dry, "identity": identity,
            "identity_sha256": canonical_sha256(identity), "required_additional_bytes": storage,
            "retention_forecast": forecast,
            "retention_scope": ("final, initial and all metadata retained; completed milestone/recovery payloads "
                                "deleted after evaluation" if prune else "all completed stage artifacts retained"),
            "comparison_pairs": [{"reference": reference_candidate, "candidate": t["name"]}
                                 for t in trajectories if t["name"] != reference_candidate],
            "runtime_cap_based_usd": total("runtime_cap_based_usd"),
            "reservation_cap_based_usd": total("reservation_cap_based_usd"),
            "scope": "full configured schedule plus optional cooldown and evaluation stages; no final test",
            "cost_scope": "cap-based estimates; each stage admits and bills its actual elapsed time"}


# ====================================================================================== the journal
class _Journal:
    """``sweep.json``: the frozen plan plus one record per stage, rewritten durably after every
    change of state."""

    def __init__(self, out: Path, planned: dict):
        self.out, self.path = out, out / "sweep.json"
        identity, digest = planned["identity"], planned["identity_sha256"]
        self.sources = identity["runtime_source_sha256"]
        if self.path.exists():
            self.data = json.loads(self.path.read_text())
            if self.data.get("identity_sha256") != digest or self.data.get("identity") != identity:
                raise ValueError("frozen sweep identity mismatch")
            if any(s["status"] != "complete" for s in self.data["stages"].values()):
                raise RuntimeError("interrupted/failed sweep stage requires explicit recovery; automatic retry forbidden")
        else:
            if any(p.name != ".sweep.lock" for p in out.iterdir()):
                raise FileExistsError("sweep output contains unjournaled artifacts")
            self.data = {**planned, "stages": {}, "prune_operations": {}, "status": "pending"}
            self.save()

    @property
    def stages(self) -> dict:
        return self.data["stages"]

    def save(self):
        write_json(self.path, self.data)

    def check_sources(self):
        if _sources() != self.sources:
            raise ValueError("frozen runtime sources changed during sweep")

    def _pruned(self, key, present) -> set:
        """Artifacts of stage ``key`` that a prune operation removed (so may be missing)."""
        gone = set()
        for op in self.data.get("prune_operations", {}).values():
            for item in op["files"].values():
                if item["stage"] != key:
                    continue
                if item["artifact"] not in present:
                    gone.add(item["artifact"])
                elif op["status"] == "complete":
                    raise ValueError("completed prune payload unexpectedly reappeared")
        return gone

    def verify(self, key, directory, ledger=None):
        """The result of a completed stage after re-hashing its artifacts and billing."""
        record = self.stages[key]
        reject_symlink_chain(self.out, directory)
        present = _artifacts(directory)
        expected = {k: v for k, v in record["artifacts"].items() if k not in self._pruned(key, present)}
        if present != expected:
            raise ValueError(f"completed stage artifact hash mismatch: {key}")
        if json.loads((Path(directory) / _STAGE_RESULT).read_text()) != record["result"]:
            raise ValueError("cached stage result differs from frozen artifact")
        if ledger is not None and _terminal_billing(ledger, directory) != record["billing"]:
            raise ValueError("completed stage billing identity changed")
        return record["result"]

    def stage(self, key, directory, produce: Callable[[], dict], ledger=None):
        """Run stage ``key`` (or re-verify it if already complete); journals running, complete or
        failed, never retrying a failure."""
        directory = Path(directory)
        if key in self.stages:
            return self.verify(key, directory, ledger)
        if directory.exists():
            raise FileExistsError(f"unjournaled stage output: {directory}")
        self.stages[key] = {"status": "running"}
        self.data["status"] = "running"
        self.save()
        try:
            result = produce()
            self.check_sources()
            billing = _terminal_billing(ledger, directory) if ledger is not None else None
            write_json(directory / _STAGE_RESULT, result)
            self.stages[key] = {"status": "complete", "artifacts": _artifacts(directory), "result": result,
                                "billing": billing}
            self.save()
            return result
        except BaseException as exc:
            self.stages[key] = {"status": "failed", "error": f"{type(exc).__name__}: {exc}"}
            self.data["status"] = "failed"
            self.save()
            raise


# ====================================================================================== the stages
class _Sweep:
    def __init__(self, out: Path, planned: dict, journal: _Journal, *, max_seconds, evaluation_max_seconds,
                 max_prediction_tokens, bootstrap_samples, prune: bool):
        self.out, self.journal = out, journal
        self.trajectories = planned["identity"]["trajectories"]
        self.controls = planned["identity"]["controls"]
        self.canary = self.controls["throughput_canary"]
        self.cooldown = self.controls["cooldown"]
        self.max_seconds, self.evaluation_max_seconds = max_seconds, evaluation_max_seconds
        self.max_prediction_tokens, self.bootstrap_samples = max_prediction_tokens, bootstrap_samples
        self.prune_enabled = prune

    def _check_inputs(self, run):
        self.journal.check_sources()
        for item in run["data"].values():
            if file_sha256(item["path"]) != item["sha256"]:
                raise ValueError("frozen data manifest changed before stage")

    @staticmethod
    def _ledger(run) -> str:
        return run["config"]["project"]["spend_ledger"]

    # ------------------------------------------------------------------ disk admission
    def admit_remaining(self):
        """Reserve disk for the training stages not yet journaled."""
        stages = self.journal.stages
        if self.prune_enabled:
            forecast = retention_forecast(self.trajectories, stages)
            self.journal.data["pending_retention_forecast"] = forecast
            pending = forecast["required_additional_bytes"]
        else:
            pending = 0
            for t in self.trajectories:
                if f"{t['name']}/parent" not in stages:
                    pending += t["parent_storage_plan"]["required_additional_bytes"]
                if t["cooldown_storage_plan"] and f"{t['name']}/cooldown" not in stages:
                    pending += t["cooldown_storage_plan"]["required_additional_bytes"]
        self.journal.data["disk_admission"] = require_checkpoint_space(self.out, pending)
        self.journal.save()

    # ------------------------------------------------------------------ per candidate
    def parent(self, run, cfg, directory: Path) -> dict:
        from .throughput_canary import ThroughputCanary
        self._check_inputs(run)
        canary = self.canary
        observer = (ThroughputCanary(canary["measured_steps"], canary["min_tokens_per_second"], canary["warmup_steps"])
                    if canary else None)
        result = train_run(cfg, directory, max_steps=run["parent_steps"], max_seconds=self.max_seconds,
                           device=self.controls["device"], **({"_throughput_canary": observer} if observer else {}))
        if Path(result["checkpoint"]).resolve() != (directory / "final").resolve():
            raise ValueError("parent returned checkpoint outside expected final directory")
        data_hash = run["data"]["training"]["sha256"]
        final = _gate_checkpoint(result["checkpoint"], run["config"], run["tokens"], manifest_hash=data_hash)
        branch = (_gate_checkpoint(directory / f"milestone-{run['branch_threshold']:012d}", run["config"],
                                   run["branch_tokens"], manifest_hash=data_hash) if self.cooldown else None)
        return {"checkpoint": final, "branch": branch, **({"throughput_canary": observer.report()} if observer else {})}

    def cooled(self, run, cfg, directory: Path, parent: dict) -> dict:
        self._check_inputs(run)
        branch = parent["branch"]
        result = train_run(cfg, directory, max_steps=run["cooldown_steps"], max_seconds=self.max_seconds,
                           device=self.controls["device"], resume=branch["path"], cooldown_steps=run["cooldown_steps"],
                           cooldown_end_tokens=run["tokens"])
        if Path(result["checkpoint"]).resolve() != (directory / "final").resolve():
            raise ValueError("cooldown returned checkpoint outside expected final directory")
        return _gate_checkpoint(result["checkpoint"], run["config"], run["tokens"], cooldown_steps=run["cooldown_steps"],
                                manifest_hash=run["data"]["training"]["sha256"],
                                parent={"path": branch["path"], "manifest_sha256": branch["manifest_sha256"]})

    def evaluation(self, run, cfg, directory: Path, selected: dict) -> dict:
        self._check_inputs(run)
        report = evaluate_checkpoint(cfg, selected["path"], directory, context=self.controls["evaluation_context"],
                                     max_prediction_tokens=self.max_prediction_tokens,
                                     max_seconds=self.evaluation_max_seconds, device=self.controls["device"],
                                     bootstrap_samples=self.bootstrap_samples)
        if (report.get("kind") != "held_out_validation" or not report["frozen_state"]["unchanged"]
                or report["validation_manifest_sha256"] != run["data"]["validation"]["sha256"]
                or report["checkpoint_manifest_sha256"] != selected["manifest_sha256"]
                or report["checkpoint_state_sha256"] != selected["state_sha256"]):
            raise ValueError("evaluation protocol/state mismatch")
        return {k: report[k] for k in ("checkpoint_manifest_sha256", "checkpoint_state_sha256",
                                       "validation_manifest_sha256", "target_plan_sha256",
                                       "available_prefix_plan_sha256", "prediction_tokens", "ce")}

    def candidate(self, run):
        """Parent, optional cooldown and evaluation of one candidate; returns (training directories,
        evaluation summary)."""
        name, cfg, ledger = run["name"], _config(run["config"]), self._ledger(run)
        parent_dir = self.out / name / "parent"
        parent = self.journal.stage(f"{name}/parent", parent_dir, lambda: self.parent(run, cfg, parent_dir), ledger)
        dirs, selected = [parent_dir], parent["checkpoint"]
        if self.cooldown:
            cooled_dir = self.out / name / "cooldown"
            selected = self.journal.stage(f"{name}/cooldown", cooled_dir,
                                          lambda: self.cooled(run, cfg, cooled_dir, parent), ledger)
            dirs.append(cooled_dir)
        eval_dir = self.out / name / "evaluation"
        summary = self.journal.stage(f"{name}/evaluation", eval_dir,
                                     lambda: self.evaluation(run, cfg, eval_dir, selected), ledger)
        return dirs, {"name": name, **summary}

    # ------------------------------------------------------------------ pruning
    def _prunable(self, run) -> dict:
        files = {}
        for phase in ("parent", "cooldown"):
            key = f"{run['name']}/{phase}"
            for rel, info in self.journal.stages.get(key, {}).get("artifacts", {}).items():
                if intermediate_payload(rel):
                    files[f"{key}/{rel}"] = {"stage": key, "artifact": rel, **info}
        return files

    def prune(self, run):
        """Delete the candidate's milestone/recovery payloads: verify its stages, refuse while a
        live run pins one, journal the plan, then unlink (resumable if interrupted)."""
        ledger = Path(self._ledger(run))
        with Path(str(ledger) + ".lock").open("a") as ledger_lock:  # the ledger's own admission lock
            fcntl.flock(ledger_lock, fcntl.LOCK_EX)
            keys = [f"{run['name']}/parent", f"{run['name']}/evaluation"]
            if run["cooldown_storage_plan"] is not None:
                keys.append(f"{run['name']}/cooldown")
            for key in keys:
                self.journal.verify(key, self.out / key, ledger)
            slated = {str((self.out / rel).parent) for rel in self._prunable(run)}
            own = {str(self.out / k) for k in keys}
            for run_id, row in json.loads(ledger.read_text())["runs"].items():
                pinned = row.get("parent_checkpoint")
                if (run_id not in own and pinned is not None and str(Path(pinned).resolve()) in slated
                        and (row.get("status") != "complete" or row.get("reserved_usd") != 0)):
                    raise ValueError("an active run pins a slated checkpoint payload")
            operations = self.journal.data.setdefault("prune_operations", {})
            if run["name"] not in operations:
                files = self._prunable(run)
                operations[run["name"]] = {"status": "planned", "files": files,
                                           "original_payload_bytes": sum(i["bytes"] for i in files.values())}
                self.journal.save()  # durable authorisation before any unlink
            op = operations[run["name"]]
            if op["status"] != "complete":
                for rel, item in op["files"].items():
                    unlink_payload(self.out, rel, item)
                op["status"] = "complete"
                self.journal.save()

    # ------------------------------------------------------------------ across candidates
    def comparisons(self, reports) -> list:
        if len({(r["target_plan_sha256"], r["available_prefix_plan_sha256"], r["prediction_tokens"])
                for r in reports}) != 1:
            raise ValueError("candidate validation targets/prefixes differ; comparison rejected")
        ref = self.controls["reference_candidate"]
        out = []
        for run in self.trajectories:
            if run["name"] == ref:
                continue
            cdir = self.out / "comparisons" / run["name"]

            def compare(run=run, cdir=cdir):
                report = compare_evaluations(self.out / ref / "evaluation" / "evaluation.json",
                                             self.out / run["name"] / "evaluation" / "evaluation.json", cdir,
                                             bootstrap_samples=self.bootstrap_samples,
                                             seed=self.controls["comparison_seed"])
                return {"reference_candidate": ref, "candidate": run["name"], "path": str(cdir / "comparison.json"),
                        "delta_ce_right_minus_left": report["delta_ce_right_minus_left"],
                        "delta_ce_95_ci": report["uncertainty"]["delta_ce_95_ci"],
                        "uncertainty": report["uncertainty"], "training_comparison": report["training_comparison"]}
            out.append(self.journal.stage(f"comparison/{run['name']}", cdir, compare))
        return out

    def summary(self, training_dirs, reports, comparisons):
        sdir = self.out / "summary"

        def summarize():
            result = summarize_runs(training_dirs, sdir)
            write_json(sdir / "validation.json", {"evaluations": reports,
                                                  "reference_candidate": self.controls["reference_candidate"],
                                                  "comparisons": comparisons, "automatic_ranking_eligible": False,
                                                  "scope": "validation only; one seed per candidate; no promotion"})
            return result
        self.journal.stage("summary", sdir, summarize)

    def run(self) -> dict:
        operations = self.journal.data.get("prune_operations", {})
        for run in self.trajectories:  # finish deletions an interrupted invocation had authorised
            if operations.get(run["name"], {}).get("status") == "planned":
                self.prune(run)
        if self.journal.data["status"] != "complete":
            self.admit_remaining()
        training_dirs, reports = [], []
        for run in self.trajectories:
            dirs, report = self.candidate(run)
            training_dirs += dirs
            reports.append(report)
            if self.prune_enabled:
                self.prune(run)
        self.summary(training_dirs, reports, self.comparisons(reports))
        self.journal.data["status"] = "complete"
        self.journal.save()
        return self.journal.data


def _canary_controls(canary_steps, min_tokens_per_second, canary_warmup_steps):
    from .throughput_canary import ThroughputCanary
    if type(canary_steps) is not int or canary_steps < 0:
        raise ValueError("canary_steps must be a nonnegative integer")
    if not canary_steps:
        if min_tokens_per_second is not None or canary_warmup_steps != 12:
            raise ValueError("canary threshold/warmup requires positive canary_steps")
        return None
    ThroughputCanary(canary_steps, min_tokens_per_second, canary_warmup_steps)  # validates the controls
    return {"measured_steps": canary_steps, "min_tokens_per_second": min_tokens_per_second,
            "warmup_steps": canary_warmup_steps,
            "scope": "first measured parent updates after the excluded warm-up; no extra trajectory"}


def run_sweep(base_cfg, candidates, out_dir, *, max_seconds, evaluation_max_seconds, device="cuda", cooldown=True,
              max_prediction_tokens=1_000_000, bootstrap_samples=1000, reference_candidate=None,
              prune_completed_intermediates=False, canary_steps=0, min_tokens_per_second=None, canary_warmup_steps=12):
    """Plan the sweep (returned as is for a dry run), then run or resume it in ``out_dir``."""
    canary = _canary_controls(canary_steps, min_tokens_per_second, canary_warmup_steps)
    if type(prune_completed_intermediates) is not bool:
        raise ValueError("prune_completed_intermediates must be Boolean")
    for cap in (max_seconds, evaluation_max_seconds):
        if isinstance(cap, bool) or not isinstance(cap, (int, float)) or not math.isfinite(cap) or cap <= 0:
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
    out.mkdir(parents=True, exist_ok=True)
    with (out / ".sweep.lock").open("a") as lock:
        try:
            fcntl.flock(lock, fcntl.LOCK_EX | fcntl.LOCK_NB)
        except BlockingIOError as exc:
            raise RuntimeError("another sweep invocation holds the output lock") from exc
        sweep = _Sweep(out, planned, _Journal(out, planned), max_seconds=max_seconds,
                       evaluation_max_seconds=evaluation_max_seconds, max_prediction_tokens=max_prediction_tokens,
                       bootstrap_samples=bootstrap_samples, prune=prune_completed_intermediates)
        return sweep.run()
