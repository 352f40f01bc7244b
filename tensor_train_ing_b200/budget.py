"""The spend ledger: locked admission and accounting of a project's compute dollars.

One JSON file (``{"version": 1, "runs": {id: row}}``) records every run and external charge.  Runs
reserve their worst-case cost (hourly rate x runtime cap x (1 + margin)) before they start, so jobs
starting in parallel cannot allocate the same dollars; a finished run replaces its reservation by
its measured cost.  Admission holds three limits: the project total, the project total less the
reserve for every stage but "Reserve", and the run's stage budget.  A crashed run keeps its
reservation until an operator reconciles it against explicit evidence.

The file, its lock (``<ledger>.lock``, an exclusive ``flock`` for writers, shared for readers) and
the row schema are the reference's (tnlm/budget.py:18-217), so runs of either framework book into
one ledger.
"""
from __future__ import annotations

import contextlib
import copy
import fcntl
import hashlib
import json
import math
from pathlib import Path

from .durable import write_json
from .hashing import canonical_sha256

STAGE_BUDGETS = {"A": 150.0, "B": 175.0, "C": 175.0, "D": 350.0, "Reserve": 150.0}
UNRESOLVED = ("running", "reconciled_unknown_tail")


def _finite_nonnegative(*values) -> bool:
    return all(not isinstance(v, bool) and isinstance(v, (int, float)) and math.isfinite(v) and v >= 0
               for v in values)


def _allocated(rows, stage=None, exclude_stage=None) -> float:
    """Spent plus reserved dollars over the rows (optionally of one stage, or all but one)."""
    total = 0.0
    for row in rows:
        s = row.get("stage", "A")
        if (stage is None or s == stage) and (exclude_stage is None or s != exclude_stage):
            total += row.get("spent_usd", 0) + row.get("reserved_usd", 0)
    return total


def read_evidence(run_id, paths) -> tuple[list, float]:
    """Metrics files an operator supplies for a reconciliation: each is fingerprinted, every record
    must name this run if it names one, and the largest ``run_elapsed_seconds`` is the observed
    lower bound of the run's elapsed time.  JSON (an object or a list) or JSON lines."""
    target = str(Path(run_id).resolve())
    evidence, elapsed = [], 0.0
    for name in paths:
        path = Path(name).resolve()
        blob = path.read_bytes()
        try:
            parsed = json.loads(blob)
            records = parsed if isinstance(parsed, list) else [parsed]
        except json.JSONDecodeError:  # JSON lines; a torn line fails the whole reconciliation
            records = [json.loads(line) for line in blob.splitlines() if line.strip()]
        named = True
        for rec in records:
            if not isinstance(rec, dict):
                raise ValueError(f"{path}: every evidence record must be a JSON object")
            who = rec.get("run_id", rec.get("run_dir"))
            if who is None:
                named = False
            elif str(Path(who).resolve()) != target:
                raise ValueError(f"{path}: evidence belongs to another run ({who})")
            seconds = rec.get("run_elapsed_seconds")
            if seconds is not None:
                if not _finite_nonnegative(seconds):
                    raise ValueError(f"{path}: run_elapsed_seconds must be a finite nonnegative number")
                elapsed = max(elapsed, float(seconds))
        evidence.append({"path": str(path), "sha256": hashlib.sha256(blob).hexdigest(), "bytes": len(blob),
                         "identity_verified": named})
    return evidence, elapsed


class SpendLedger:
    def __init__(self, path, total_budget=1000.0, reserve=150.0, stage_budgets=None):
        self.path = Path(path)
        self.total, self.reserve = float(total_budget), float(reserve)
        if not (math.isfinite(self.total) and math.isfinite(self.reserve) and 0 <= self.reserve <= self.total):
            raise ValueError("the project budget and reserve must be finite with 0 <= reserve <= total")
        if stage_budgets is not None and (not isinstance(stage_budgets, dict) or set(stage_budgets) - set(STAGE_BUDGETS)):
            raise ValueError(f"stage budgets may only name the stages {sorted(STAGE_BUDGETS)}")
        merged = {**STAGE_BUDGETS, **(stage_budgets or {})}
        self.stage_budgets = {k: float(v) for k, v in merged.items()}
        if not _finite_nonnegative(*self.stage_budgets.values()):
            raise ValueError("stage budgets must be finite and nonnegative")
        self.stage_budgets["Reserve"] = min(self.reserve, self.stage_budgets["Reserve"])

    # ------------------------------------------------------------------ storage
    @property
    def _lock_path(self) -> str:
        return str(self.path) + ".lock"

    @contextlib.contextmanager
    def locked(self):
        """The ledger contents for a read-modify-write under the exclusive lock; written back
        durably when the block completes."""
        self.path.parent.mkdir(parents=True, exist_ok=True)
        with open(self._lock_path, "a") as lock:
            fcntl.flock(lock, fcntl.LOCK_EX)
            data = json.loads(self.path.read_text()) if self.path.exists() else {"version": 1, "runs": {}}
            yield data
            write_json(self.path, data, indent=2)

    def _snapshot(self) -> dict:
        with open(self._lock_path, "a") as lock:
            fcntl.flock(lock, fcntl.LOCK_SH)
            return json.loads(self.path.read_text())

    # ------------------------------------------------------------------ runs
    def _admit(self, rows: dict, stage: str, amount: float) -> None:
        everything = rows.values()
        if _allocated(everything) + amount > self.total:
            raise ValueError("project budget exhausted (including reserve and active runs)")
        if stage != "Reserve" and _allocated(everything, exclude_stage="Reserve") + amount > self.total - self.reserve:
            raise ValueError("project budget exhausted (including reserve and active runs)")
        if _allocated(everything, stage=stage) + amount > self.stage_budgets[stage]:
            raise ValueError(f"stage {stage} budget exhausted")

    def begin(self, run_id, hourly_rate, max_seconds, run_budget=None, *, parent_checkpoint=None,
              cost_margin_fraction=0.0, stage="A"):
        """Reserve a run's worst-case cost; returns the reserved dollars."""
        if stage not in self.stage_budgets:
            raise ValueError(f"unknown budget stage: {stage}")
        rate, seconds, margin = float(hourly_rate), float(max_seconds), float(cost_margin_fraction)
        if not (_finite_nonnegative(rate, seconds) and seconds > 0):
            raise ValueError("a run needs a finite nonnegative hourly rate and a positive runtime cap")
        if not _finite_nonnegative(margin):
            raise ValueError("the cost margin must be finite and nonnegative")
        amount = rate * seconds / 3600 * (1 + margin)
        if run_budget is not None and (not math.isfinite(run_budget) or amount > run_budget):
            raise ValueError("the runtime reservation exceeds the run budget")
        with self.locked() as data:
            if run_id in data["runs"]:
                raise ValueError(f"duplicate run ID: {run_id}")
            self._admit(data["runs"], stage, amount)
            data["runs"][run_id] = {"status": "running", "rate_usd_per_hour": rate, "reserved_usd": amount,
                                    "spent_usd": 0.0,
                                    "parent_checkpoint": str(Path(parent_checkpoint).resolve()) if parent_checkpoint
                                    else None,
                                    "cost_margin_fraction": margin, "stage": stage, "kind": "runtime"}
        return amount

    def finish(self, run_id, elapsed, status):
        """Replace a running reservation by the measured cost of ``elapsed`` seconds."""
        with self.locked() as data:
            row = data["runs"][run_id]
            if row["status"] != "running":
                raise ValueError("only a running reservation can be finished")
            row.update(status=status, elapsed_seconds=elapsed, spent_usd=elapsed * row["rate_usd_per_hour"] / 3600,
                       reserved_usd=0.0)

    def record_charge(self, charge_id, usd, *, stage="Reserve", description):
        """Book an external charge that was already paid: recorded even beyond a cap (the overrun stays
        visible and blocks later admissions).  Nothing external is called."""
        usd = float(usd)
        if stage not in self.stage_budgets or not _finite_nonnegative(usd) or not description:
            raise ValueError("a charge needs a known stage, a finite nonnegative amount and a description")
        with self.locked() as data:
            if charge_id in data["runs"]:
                raise ValueError(f"duplicate run/charge ID: {charge_id}")
            row = {"kind": "external", "status": "charged", "stage": stage, "spent_usd": usd, "reserved_usd": 0.0,
                   "description": description}
            data["runs"][charge_id] = row
            rows = data["runs"].values()
            row["exceeds_project_budget"] = _allocated(rows) > self.total
            row["exceeds_stage_budget"] = _allocated(rows, stage=stage) > self.stage_budgets[stage]
        return row

    # ------------------------------------------------------------------ reconciliation
    @staticmethod
    def _row_digest(row) -> str:
        return canonical_sha256(row)

    @staticmethod
    def _require_unresolved(row):
        if row.get("kind", "runtime") != "runtime" or row["status"] not in UNRESOLVED:
            raise ValueError("only unresolved runtime entries can be reconciled")

    def inspect_reconciliation(self, run_id, *, evidence_paths=()):
        """What a reconciliation of ``run_id`` would start from, read without writing the ledger:
        the row and its digest (to pin in ``reconcile_terminal``) and the evidence's lower bound.
        Metrics bound the elapsed time from below; they never prove the job stopped."""
        row = copy.deepcopy(self._snapshot()["runs"][run_id])
        self._require_unresolved(row)
        evidence, elapsed = read_evidence(run_id, evidence_paths)
        return {"run_id": run_id, "row": row, "row_sha256": self._row_digest(row), "evidence": evidence,
                "observed_elapsed_seconds": elapsed,
                "observed_cost_lower_bound_usd": max(row.get("spent_usd", 0.0), elapsed * row["rate_usd_per_hour"] / 3600),
                "termination_verified": False, "tail_cost_known": False}

    def reconcile_terminal(self, run_id, *, expected_row_sha256, operator, reason, terminal_attestation,
                           observed_elapsed_seconds=None, total_elapsed_seconds=None, total_cost_usd=None,
                           evidence_paths=()):
        """Operator bookkeeping for a run that stopped without finishing its row.

        ``terminal_attestation`` must be exactly ``{"run_id": run_id, "all_workers_stopped": True}``.
        With a known total (elapsed seconds or dollars) the reservation is released; with only a
        lower bound the row keeps its original allocation as spent + reserved.  An audit entry is
        appended; no process or provider is contacted and completion of training is never inferred."""
        if terminal_attestation != {"run_id": run_id, "all_workers_stopped": True}:
            raise ValueError("an explicit terminal attestation naming this run is required")
        if not (isinstance(operator, str) and operator.strip() and isinstance(reason, str) and reason.strip()):
            raise ValueError("an operator and a reason are required")
        given = [v for v in (observed_elapsed_seconds, total_elapsed_seconds, total_cost_usd) if v is not None]
        if not _finite_nonnegative(*given):
            raise ValueError("reconciliation amounts must be finite and nonnegative")
        if total_elapsed_seconds is not None and total_cost_usd is not None:
            raise ValueError("give one authoritative total: elapsed seconds or dollars")
        evidence, elapsed = read_evidence(run_id, evidence_paths)
        elapsed = max(elapsed, observed_elapsed_seconds or 0.0)
        with self.locked() as data:
            row = data["runs"][run_id]
            if self._row_digest(row) != expected_row_sha256:
                raise ValueError("the ledger row changed since it was inspected")
            self._require_unresolved(row)
            before = copy.deepcopy(row)
            for earlier in row.get("reconciliations", []):
                elapsed = max(elapsed, earlier.get("observed_elapsed_seconds", 0.0))
            rate = row["rate_usd_per_hour"]
            floor = max(row.get("spent_usd", 0.0), elapsed * rate / 3600)
            total = total_cost_usd
            if total_elapsed_seconds is not None:
                if total_elapsed_seconds < elapsed:
                    raise ValueError("the total elapsed time is below the observed lower bound")
                total = total_elapsed_seconds * rate / 3600
            if total is not None and total < floor:
                raise ValueError("the total cost is below the observed lower bound")
            if not math.isfinite(floor) or (total is not None and not math.isfinite(total)):
                raise ValueError("the reconciled cost overflowed")
            known = total is not None
            held = row.get("spent_usd", 0.0) + row.get("reserved_usd", 0.0)
            row.update(status="reconciled_terminal" if known else "reconciled_unknown_tail",
                       spent_usd=total if known else floor, reserved_usd=0.0 if known else max(0.0, held - floor))
            row.setdefault("reconciliations", []).append({
                "operator": operator, "reason": reason, "terminal_attestation": copy.deepcopy(terminal_attestation),
                "old_row": before, "old_row_sha256": expected_row_sha256, "observed_elapsed_seconds": elapsed,
                "total_elapsed_seconds": total_elapsed_seconds, "total_cost_usd": total_cost_usd,
                "tail_cost_known": known, "evidence": evidence})
            result, digest = copy.deepcopy(row), self._row_digest(row)
        return {"run_id": run_id, "row": result, "row_sha256": digest, "tail_cost_known": known,
                "training_completion_verified": False}
