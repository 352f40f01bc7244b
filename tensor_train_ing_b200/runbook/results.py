"""Experiment-result tools over run directories (the roles of the reference's fit_lr_optimum.py,
check_contamination.py, find_orphan_states.py and export_results.py in tnlm ``scripts/``).

    python -m tensor_train_ing_b200.runbook.results lr-optimum runs/ --pattern 'w(?P<group>\\d+)_lr(?P<lr>[0-9.e-]+)'
    python -m tensor_train_ing_b200.runbook.results contamination --train DATA_DIR [--val DATA_DIR] [--n 13]
    python -m tensor_train_ing_b200.runbook.results states runs/ [--min-age-min 30] [--keep SUBSTRING ...]
    python -m tensor_train_ing_b200.runbook.results export runs/ results/ [--max-rows 400]

* ``lr-optimum``: every ``evaluation/evaluation.json`` whose candidate directory name matches the
  pattern (named groups ``group`` and ``lr``; with ``--descriptor-lr`` the rate comes from the
  report's training descriptor) gives one CE per (group, lr), the newest file winning.  Per group
  with three or more rates, CE is fitted as a parabola in log(lr): its vertex is the optimum,
  flagged as extrapolated outside the sampled range and as unidentifiable when the CE spread is
  below ``--flat``; when the best sampled rate is an end point the next rate to bracket it is
  suggested.  Groups that are integers (widths) with interior optima give a power law
  optimum = k * group**slope.
* ``contamination``: the share of each validation document's ``n``-token windows that occur in an
  evenly spaced sample of the training split (windows hashed with a 64-bit polynomial rolling
  hash, so collisions are negligible at these sizes).  The held-out exclusion removes exact copies;
  this finds near-duplicates.  Documents at or above ``--flag`` are listed; exit status 1 if any.
* ``states``: checkpoint payloads (``state.pt``) whose run already holds an evaluation, older than
  ``--min-age-min`` and outside ``--keep``, with their sizes: candidates for deletion (nothing is
  deleted).
* ``export``: a small mirror without weights: per run ``curve.json`` (step, tokens, loss, lr,
  grad_norm, evenly thinned to ``--max-rows`` with the last row kept, plus every QK-clip and
  stability record) and ``evaluation.json`` (CE, interval, descriptor, per-document sums).
  Unchanged outputs are not rewritten.
"""
from __future__ import annotations

import argparse
import json
import math
import re
import sys
import time
from pathlib import Path

import numpy as np

FLAT_CE = 0.015


# ------------------------------------------------------------------------------------ LR optimum
def collect_lr_points(runs, pattern: str, *, extra=(), exclude: str | None = None,
                      descriptor_lr: bool = False) -> dict:
    """{group: {lr: ce}} from the evaluations under ``runs`` whose candidate name matches."""
    runs = Path(runs)
    matchers = [re.compile(p) for p in (pattern, *extra)]
    skip = re.compile(exclude) if exclude else None
    newest: dict = {}
    for report in runs.rglob("evaluation/evaluation.json"):
        if skip is not None and skip.search(str(report.relative_to(runs))):
            continue
        name = report.parent.parent.name
        hit = next((m for m in (r.fullmatch(name) for r in matchers) if m), None)
        if hit is None:
            continue
        data = json.loads(report.read_text())
        group = hit.group("group")
        group = int(group) if group.isdigit() else group
        lr = float(data["training_descriptor"]["lr"]) if descriptor_lr else float(hit.group("lr"))
        stamp = report.stat().st_mtime
        if (group, lr) not in newest or stamp > newest[(group, lr)][1]:
            newest[(group, lr)] = (float(data["ce"]), stamp)
    points: dict = {}
    for (group, lr), (ce, _) in newest.items():
        points.setdefault(group, {})[lr] = ce
    return points


def fit_lr_optimum(points: dict, flat: float = FLAT_CE) -> dict:
    """Per group: sampled rates and CEs, the parabola's optimum (None without a minimum or with fewer
    than three rates), its CE, whether it is inside the sampled range, whether the CE spread is too
    flat to identify it, and the next rate that would bracket an end-point minimum."""
    out = {}
    for group in sorted(points, key=str):
        rates = sorted(points[group])
        ces = [points[group][r] for r in rates]
        row = {"lrs": rates, "ce": ces, "optimum": None, "optimum_ce": None, "interior": False,
               "flat": False, "next_lr": None}
        best = int(np.argmin(ces)) if ces else None
        if len(rates) >= 2 and best in (0, len(rates) - 1):
            row["next_lr"] = rates[0] / 2 if best == 0 else rates[-1] * 2
        if len(rates) >= 3:
            x = np.log(np.asarray(rates))
            a, b, c = np.polyfit(x, np.asarray(ces), 2)
            if a > 0:
                vertex = -b / (2 * a)
                row["optimum"] = float(math.exp(vertex))
                row["optimum_ce"] = float(c - b * b / (4 * a))
                row["interior"] = rates[0] <= row["optimum"] <= rates[-1]
            row["flat"] = max(ces) - min(ces) < flat
        out[group] = row
    return out


def optimum_power_law(fits: dict) -> dict | None:
    """log(optimum) = log(k) + slope * log(group) over integer groups with interior, identifiable optima."""
    usable = [(g, f["optimum"]) for g, f in fits.items()
              if isinstance(g, int) and f["interior"] and not f["flat"]]
    if len(usable) < 2:
        return None
    slope, intercept = np.polyfit(np.log([g for g, _ in usable]), np.log([o for _, o in usable]), 1)
    return {"slope": float(slope), "k": float(math.exp(intercept)), "groups": [g for g, _ in usable]}


# --------------------------------------------------------------------------------- contamination
_MULT = np.uint64(0x100000001B3)


def window_hashes(tokens: np.ndarray, n: int) -> np.ndarray:
    """64-bit polynomial hashes of every ``n``-token window of ``tokens`` (empty when shorter)."""
    t = np.asarray(tokens, dtype=np.uint64)
    if len(t) < n:
        return np.empty(0, dtype=np.uint64)
    h = np.zeros(len(t) - n + 1, dtype=np.uint64)
    with np.errstate(over="ignore"):
        for k in range(n):
            h = h * _MULT + t[k:len(t) - n + 1 + k] + np.uint64(1)
    return h


def _split_docs(root: Path, split: str):
    """(id, tokens) of every document of ``split`` in a prepared dataset."""
    from ..token_format import read_split_tokens
    tokens = read_split_tokens(root, split)
    with (root / "documents.jsonl").open() as fh:
        for line in fh:
            row = json.loads(line)
            if row["split"] == split:
                yield row["id"], tokens[row["token_start"]:row["token_end"]]


def contamination(train_root, val_root=None, *, n: int = 13, sample_tokens: int = 600_000_000,
                  chunk_tokens: int = 1 << 20, flag: float = 0.5) -> dict:
    """Per validation document, the share of its ``n``-grams seen in a sample of the training split."""
    from ..token_format import read_split_tokens
    train_root = Path(train_root)
    val_root = Path(val_root) if val_root is not None else train_root
    train = read_split_tokens(train_root, "train")
    take = min(len(train), int(sample_tokens))
    pieces = max(1, math.ceil(take / chunk_tokens))
    starts = np.linspace(0, max(0, len(train) - chunk_tokens), pieces).astype(np.int64) if take < len(train) else \
        np.arange(0, len(train), chunk_tokens)
    seen = np.unique(np.concatenate([window_hashes(train[s:s + chunk_tokens], n) for s in starts]
                                    or [np.empty(0, dtype=np.uint64)]))
    docs = []
    for doc_id, toks in _split_docs(val_root, "val"):
        h = window_hashes(toks, n)
        if len(h):
            docs.append({"id": doc_id, "windows": int(len(h)), "overlap": float(np.isin(h, seen).mean())})
    flagged = sorted((d for d in docs if d["overlap"] >= flag), key=lambda d: -d["overlap"])
    return {"n": n, "sampled_train_tokens": int(min(len(train), len(starts) * chunk_tokens)),
            "train_tokens": int(len(train)), "validation_documents": len(docs),
            "mean_overlap": float(np.mean([d["overlap"] for d in docs])) if docs else 0.0,
            "flag": flag, "flagged": flagged}


# ------------------------------------------------------------------------------ evaluated states
def _evaluated(run: Path) -> bool:
    return (run / "evaluation" / "evaluation.json").is_file() or any(run.glob("*.eval.json"))


def evaluated_states(runs, *, min_age_min: float = 30.0, keep=(), now: float | None = None) -> list[dict]:
    """``state.pt`` files whose run (up to three directories above) holds an evaluation."""
    now = time.time() if now is None else now
    found = []
    for state in sorted(Path(runs).rglob("state.pt")):
        if any(k in str(state) for k in keep):
            continue
        info = state.stat()
        if now - info.st_mtime < 60 * min_age_min:
            continue
        owners = [state.parents[i] for i in range(1, 4) if i < len(state.parents)]
        if any(_evaluated(p) for p in owners):
            found.append({"path": str(state), "bytes": info.st_size})
    return found


# ------------------------------------------------------------------------------------- export
def _thin(rows: list, limit: int) -> list:
    if len(rows) <= limit:
        return rows
    picks = sorted(set(np.linspace(0, len(rows) - 1, limit).round().astype(int).tolist()) | {len(rows) - 1})
    return [rows[i] for i in picks]


def _write_if_changed(path: Path, payload) -> bool:
    text = json.dumps(payload, indent=1, sort_keys=True) + "\n"
    if path.is_file() and path.read_text() == text:
        return False
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_name(path.name + ".tmp")
    tmp.write_text(text)
    tmp.replace(path)
    return True


def export_results(runs, out, *, max_rows: int = 400) -> dict:
    """Write the compact mirror of ``runs`` into ``out``; returns the files written and kept."""
    runs, out = Path(runs), Path(out)
    written, kept = [], []
    for metrics in sorted(runs.rglob("metrics.jsonl")):
        rows = [json.loads(x) for x in metrics.read_text().splitlines() if x.strip()]
        curve = [{k: r.get(k) for k in ("step", "tokens", "loss", "lr", "grad_norm")} for r in rows]
        events = [{"step": r.get("step"), **{k: r[k] for k in ("qk_clip", "stability") if k in r}}
                  for r in rows if "qk_clip" in r or "stability" in r]
        target = out / metrics.parent.relative_to(runs) / "curve.json"
        (written if _write_if_changed(target, {"rows": _thin(curve, max_rows), "logged_rows": len(rows),
                                               "events": events}) else kept).append(str(target))
    for report in sorted(runs.rglob("evaluation.json")):
        data = json.loads(report.read_text())
        if "ce" not in data:
            continue
        summary = {k: data.get(k) for k in ("ce", "prediction_tokens", "uncertainty", "training_descriptor",
                                            "model_sha256", "target_plan_sha256")}
        if "documents" in data:
            summary["documents"] = data["documents"]
        target = out / report.relative_to(runs)
        (written if _write_if_changed(target, summary) else kept).append(str(target))
    return {"written": written, "unchanged": kept}


# ----------------------------------------------------------------------------------------- CLI
def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m tensor_train_ing_b200.runbook.results")
    sub = ap.add_subparsers(dest="cmd", required=True)
    lr = sub.add_parser("lr-optimum")
    lr.add_argument("runs")
    lr.add_argument("--pattern", required=True)
    lr.add_argument("--also", nargs="*", default=[])
    lr.add_argument("--exclude")
    lr.add_argument("--descriptor-lr", action="store_true")
    lr.add_argument("--flat", type=float, default=FLAT_CE)
    ct = sub.add_parser("contamination")
    ct.add_argument("--train", required=True)
    ct.add_argument("--val")
    ct.add_argument("--n", type=int, default=13)
    ct.add_argument("--sample-tokens", type=float, default=6e8)
    ct.add_argument("--flag", type=float, default=0.5)
    st = sub.add_parser("states")
    st.add_argument("runs")
    st.add_argument("--min-age-min", type=float, default=30.0)
    st.add_argument("--keep", nargs="*", default=[])
    ex = sub.add_parser("export")
    ex.add_argument("runs")
    ex.add_argument("out")
    ex.add_argument("--max-rows", type=int, default=400)
    a = ap.parse_args(argv)
    if a.cmd == "lr-optimum":
        fits = fit_lr_optimum(collect_lr_points(a.runs, a.pattern, extra=a.also, exclude=a.exclude,
                                                descriptor_lr=a.descriptor_lr), flat=a.flat)
        print(json.dumps({"groups": {str(g): f for g, f in fits.items()}, "power_law": optimum_power_law(fits)},
                         indent=1))
        return 0
    if a.cmd == "contamination":
        report = contamination(a.train, a.val, n=a.n, sample_tokens=int(a.sample_tokens), flag=a.flag)
        print(json.dumps(report, indent=1))
        return 1 if report["flagged"] else 0
    if a.cmd == "states":
        found = evaluated_states(a.runs, min_age_min=a.min_age_min, keep=a.keep)
        print(json.dumps({"states": found, "total_bytes": sum(f["bytes"] for f in found)}, indent=1))
        return 0
    print(json.dumps(export_results(a.runs, a.out, max_rows=a.max_rows), indent=1))
    return 0


if __name__ == "__main__":
    sys.exit(main())
