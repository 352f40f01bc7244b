"""Steady-state training throughput of run directories, and regression checks against a baseline.

    python -m tensor_train_ing_b200.runbook.throughput RUN_DIR_OR_METRICS [...] [--last N]
    python -m tensor_train_ing_b200.runbook.throughput --drop METRICS           # recent / steady ratio
    python -m tensor_train_ing_b200.runbook.throughput RUN ... --baseline base.json --tolerance 0.05

The steady rate of a run is tokens over run time between the middle logged row and the last (the
first half holds start-up, kernel warm-up and early checkpoints); ``--last N`` uses the last N rows
instead (a live run).  A directory argument is searched for ``metrics.jsonl`` files (a sweep's
``parent`` runs are named after their candidate).  ``--baseline`` compares each run with the rate
recorded for its name and fails (exit 1) when one falls more than ``--tolerance`` below it;
``--record`` writes the measured rates as a new baseline.
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path


def _rows(path) -> list[dict]:
    rows = []
    for line in Path(path).read_text().splitlines():
        row = json.loads(line)
        if "run_elapsed_seconds" in row and "tokens" in row:
            rows.append(row)
    return rows


def steady_rate(path, last: int | None = None) -> float | None:
    """Tokens per second between the middle (or the last ``last``-th) row and the final row."""
    rows = _rows(path)
    if len(rows) < 4:
        return None
    first = rows[max(0, len(rows) - 1 - last)] if last else rows[len(rows) // 2]
    seconds = rows[-1]["run_elapsed_seconds"] - first["run_elapsed_seconds"]
    return (rows[-1]["tokens"] - first["tokens"]) / seconds if seconds > 0 else None


def drop_ratio(path, last: int = 20, min_rows: int = 40) -> float | None:
    """Recent rate over the steady rate: well below 1 means the run has slowed down."""
    if len(_rows(path)) < min_rows:
        return None
    recent, steady = steady_rate(path, last), steady_rate(path)
    return recent / steady if recent and steady else None


def run_name(metrics: Path) -> str:
    return metrics.parent.parent.name if metrics.parent.name == "parent" else metrics.parent.name


def find_metrics(arg) -> list[Path]:
    p = Path(arg)
    return [p] if p.is_file() else sorted(p.rglob("metrics.jsonl"))


def rates(args, last=None) -> dict[str, float | None]:
    return {run_name(m): steady_rate(m, last) for a in args for m in find_metrics(a)}


def regressions(measured: dict, baseline: dict, tolerance: float) -> list[dict]:
    """Runs whose rate fell more than ``tolerance`` (a fraction) below their baseline."""
    out = []
    for name, rate in measured.items():
        ref = baseline.get(name)
        if ref and (rate is None or rate < (1 - tolerance) * ref):
            out.append({"run": name, "tokens_per_second": rate, "baseline": ref,
                        "ratio": None if rate is None else rate / ref})
    return out


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("paths", nargs="+")
    p.add_argument("--last", type=int)
    p.add_argument("--drop", action="store_true", help="print the recent/steady ratio of one metrics file")
    p.add_argument("--baseline")
    p.add_argument("--tolerance", type=float, default=0.05)
    p.add_argument("--record", help="write the measured rates to this baseline file")
    a = p.parse_args(argv)
    if a.drop:
        ratio = drop_ratio(a.paths[0])
        print("n/a" if ratio is None else f"{ratio:.3f}")
        return 0
    measured = rates(a.paths, a.last)
    for name, rate in measured.items():
        print(f"{name:45s} {'n/a' if rate is None else f'{rate:10.0f} tok/s'}")
    if a.record:
        Path(a.record).write_text(json.dumps(measured, indent=2, sort_keys=True) + "\n")
    if a.baseline:
        bad = regressions(measured, json.loads(Path(a.baseline).read_text()), a.tolerance)
        for row in bad:
            print(f"REGRESSION {row['run']}: {row['tokens_per_second']} tok/s vs baseline {row['baseline']:.0f}")
        return 1 if bad else 0
    return 0


if __name__ == "__main__":
    sys.exit(main())
