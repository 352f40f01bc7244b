"""Run audits over directories of finished runs (the reference's check_data_epochs.py, find_runs.py
and stability_trace.py roles).

    python -m tensor_train_ing_b200.runbook.audit epochs runs/ [...]
    python -m tensor_train_ing_b200.runbook.audit find runs/ normalization=pre_rms width=2048 [--top 10]
    python -m tensor_train_ing_b200.runbook.audit stability RUN/metrics.jsonl [--jump 2.0] [--absolute 1e4]

* ``epochs``: every run whose ``result.json`` reports more input tokens read than its training split
  holds (the packed sampler wraps silently into a second epoch) is listed with its epoch count;
  exit status 1 when any is found.
* ``find``: every ``evaluation.json`` whose checkpoint's training descriptor matches all
  ``key=value`` filters (values parsed as JSON where possible), best CE first.
* ``stability``: per logged update the attention-score bound (``score_bound_max``, or the stability
  probe's maximum score), flagged where it jumps by more than ``--jump`` times the previous value,
  grows over ``--window`` consecutive rows by more than ``--runaway`` times, or exceeds
  ``--absolute``; exit status 1 when any row is flagged.
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path


def _json(path):
    try:
        return json.loads(Path(path).read_text())
    except (OSError, ValueError):
        return None


# ====================================================================================== epochs
def epoch_overreads(roots) -> list[dict]:
    found = []
    for root in roots:
        for result_path in sorted(Path(root).rglob("result.json")):
            result = _json(result_path)
            try:
                seen = int(result["progress"]["input_tokens_seen"])
                manifest = result["training_descriptor"]["configuration"]["data"]["manifest"]
                manifest = Path(manifest) / "manifest.json" if Path(manifest).is_dir() else Path(manifest)
                available = int(json.loads(manifest.read_text())["tokens"]["train"])
            except (TypeError, KeyError, ValueError, OSError):
                continue
            if seen > available:
                found.append({"run": str(result_path.parent), "input_tokens_seen": seen, "split_tokens": available,
                              "epochs": seen / available})
    return found


# ====================================================================================== find
def _parse(value: str):
    try:
        return json.loads(value)
    except ValueError:
        return value


def find_runs(roots, filters: dict) -> list[dict]:
    rows = []
    for root in roots:
        for ev_path in Path(root).rglob("evaluation.json"):
            ev = _json(ev_path)
            if not ev or ev.get("kind") != "held_out_validation":
                continue
            desc = ev.get("training_descriptor") or {}
            if all(desc.get(k) == v for k, v in filters.items()):
                rows.append({"evaluation": str(ev_path), "ce": ev["ce"], "prediction_tokens": ev["prediction_tokens"],
                             **{k: desc.get(k) for k in ("normalization", "optimizer", "width", "depth", "lr",
                                                         "actual_prediction_tokens", "completion_status")}})
    return sorted(rows, key=lambda r: r["ce"])


# ====================================================================================== stability
def _bound(row: dict):
    if row.get("score_bound_max") is not None:
        return float(row["score_bound_max"])
    stability = row.get("stability") or {}
    value = stability.get("max_score") or stability.get("score_max")
    return None if value is None else float(value)


def stability_trace(metrics, *, jump=2.0, window=20, runaway=4.0, absolute=None) -> list[dict]:
    rows = [json.loads(x) for x in Path(metrics).read_text().splitlines()]
    trace, history = [], []
    for row in rows:
        value = _bound(row)
        if value is None:
            continue
        flags = []
        if history and history[-1] > 0 and value > jump * history[-1]:
            flags.append("jump")
        if len(history) >= window and history[-window] > 0 and value > runaway * history[-window] and all(
                b >= a for a, b in zip(history[-window:], history[-window + 1:] + [value])):
            flags.append("steady_runaway")
        if absolute is not None and value > absolute:
            flags.append("absolute")
        trace.append({"step": row.get("step"), "tokens": row.get("tokens"), "score_bound": value, "flags": flags})
        history.append(value)
    return trace


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    sub = p.add_subparsers(dest="cmd", required=True)
    e = sub.add_parser("epochs")
    e.add_argument("roots", nargs="+")
    f = sub.add_parser("find")
    f.add_argument("root")
    f.add_argument("filters", nargs="*")
    f.add_argument("--top", type=int, default=20)
    s = sub.add_parser("stability")
    s.add_argument("metrics")
    s.add_argument("--jump", type=float, default=2.0)
    s.add_argument("--window", type=int, default=20)
    s.add_argument("--runaway", type=float, default=4.0)
    s.add_argument("--absolute", type=float)
    a = p.parse_args(argv)
    if a.cmd == "epochs":
        found = epoch_overreads(a.roots)
        for row in found:
            print(f"{row['run']}: read {row['input_tokens_seen']} input tokens of a {row['split_tokens']}-token split "
                  f"({row['epochs']:.2f} epochs)")
        return 1 if found else 0
    if a.cmd == "find":
        filters = dict(item.split("=", 1) for item in a.filters)
        for row in find_runs([a.root], {k: _parse(v) for k, v in filters.items()})[:a.top]:
            print(json.dumps(row))
        return 0
    trace = stability_trace(a.metrics, jump=a.jump, window=a.window, runaway=a.runaway, absolute=a.absolute)
    for row in trace:
        print(f"{row['step']:>8} {row['score_bound']:12.4g} {' '.join(row['flags'])}")
    return 1 if any(r["flags"] for r in trace) else 0


if __name__ == "__main__":
    sys.exit(main())
